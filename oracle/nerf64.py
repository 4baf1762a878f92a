"""Float64 restatement of cufk's reconstruction path: the parity oracle.

It computes on the device of its inputs: on the CPU, and, in GPU tests at full configuration
sizes, in float64 on the GPU (the same arithmetic; the sequential loop over a chain's steps is
what makes the CPU slow there).

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (``cufk_b200``) imports, calls or
executes this module; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and ``--impl reference`` legs do, and only as the checker or as the timed CPU baseline.

Parity pin: the reference ships no tests, fixtures or golden vectors.  This restatement is pinned
against the reference's own kernels, compiled for sm_100a by ``oracle/build_ref.py`` and run on a
B200: ``tests/golden/make_golden.py`` writes their outputs to ``tests/golden/*.npz`` and
``tests/test_oracle.py`` checks this module against those fixtures on the CPU.

Every function cites the reference file:line it restates (paths relative to the reference
project root).  All arithmetic is float64 torch, vectorised over the batch and sequential over
the chain, so autograd of :func:`reconstruct64` gives exact float64 gradients; the reference's
own backward formulas are restated separately in :func:`block_backward64` so both can be compared.
"""

from __future__ import annotations

import math

import torch

F64 = torch.float64

# block.cu:41 (kEps) and frame_utils.cuh:7 (kFrameEps): both are the float literal 1e-12f.
EPS = float(torch.tensor(1.0e-12, dtype=torch.float32).item())
# torsion.cu:35 (kNormEps = 1e-8f) squared in float, as clamped_pair_norm2 does (torsion.cu:119-123).
NORM_EPS2 = float(torch.tensor(1.0e-8, dtype=torch.float32).item() ** 2)
NORM_EPS2_F32 = float((torch.tensor(1.0e-8, dtype=torch.float32) * torch.tensor(1.0e-8, dtype=torch.float32)).item())

DEFAULT_P0 = (0.0, 0.0, 0.0)  # reconstruct.py:69
DEFAULT_FIRST_DIRECTION = (1.0, 0.0, 0.0)  # reconstruct.py:70
DEFAULT_INITIAL_NORMAL = (0.0, 0.0, 1.0)  # reconstruct.py:71


def _normalized(v: torch.Tensor) -> torch.Tensor:
    """frame_utils.cuh:17-20: v / sqrt(max(|v|^2, 1e-12))."""
    n2 = (v * v).sum(-1, keepdim=True)
    return v / torch.sqrt(torch.clamp(n2, min=EPS))


def _stable_perpendicular(v: torch.Tensor) -> torch.Tensor:
    """frame_utils.cuh:22-31: cross with e_x, or with e_y when |v_x| >= 0.9."""
    ex = torch.zeros_like(v)
    ex[..., 0] = 1.0
    ey = torch.zeros_like(v)
    ey[..., 1] = 1.0
    helper = torch.where((v[..., :1].abs() >= 0.9), ey, ex)
    return _normalized(torch.linalg.cross(v, helper, dim=-1))


def first_frame64(l0, l1, a0, p0, first_direction, initial_normal):
    """block.cu:113-148 (compute_first_frame), vectorised over the batch.

    ``l0, l1, a0`` are (B,) float64; anchors are (3,) float64.  Returns a dict with p1, p2, dir0,
    turn0, dir1, normal as (B, 3) and ``frame`` = [dir1 | side | normal] as (B, 3, 3) columns.
    """
    b = l0.shape[0]
    origin = p0.to(F64).expand(b, 3)
    dir0 = _normalized(first_direction.to(F64)).expand(b, 3)
    p1 = origin + l0[:, None] * dir0
    n0 = initial_normal.to(F64)
    dir0_1 = dir0[0]
    n0 = n0 - (n0 * dir0_1).sum() * dir0_1
    if float((n0 * n0).sum()) < EPS:
        n0 = _stable_perpendicular(dir0_1)
    else:
        n0 = _normalized(n0)
    turn0 = _normalized(torch.linalg.cross(n0, dir0_1, dim=-1)).expand(b, 3)
    s = torch.sin(a0)[:, None]
    c = torch.cos(a0)[:, None]
    dir1 = -c * dir0 + s * turn0
    p2 = p1 + l1[:, None] * dir1
    normal = _normalized(torch.linalg.cross(dir0, dir1, dim=-1))
    side = torch.linalg.cross(normal, dir1, dim=-1)
    frame = torch.stack([dir1, side, normal], dim=-1)  # columns (Mat3T::from_columns)
    return {"p1": p1, "p2": p2, "dir0": dir0, "turn0": turn0, "dir1": dir1, "normal": normal, "frame": frame}


def local_transform64(length, s, c, S, C):
    """affine.cuh:24-45: R rows [(-c,-s,0), (sC,-cC,-S), (sS,-cS,C)], t = length * R[:,0].

    ``s, c`` are the sine/cosine of the bond angle, ``S, C`` of the dihedral; all (B,).
    """
    zero = torch.zeros_like(s)
    rows = torch.stack(
        [
            torch.stack([-c, -s, zero], -1),
            torch.stack([s * C, -c * C, -S], -1),
            torch.stack([s * S, -c * S, C], -1),
        ],
        -2,
    )
    t = length[:, None] * torch.stack([-c, s * C, s * S], -1)
    return rows, t


def _anchors(p0, first_direction, initial_normal, device="cpu"):
    def one(x, default):
        if x is None:
            return torch.tensor(default, dtype=F64, device=device)
        return x.detach().to(device, F64)

    return (
        one(p0, DEFAULT_P0),
        one(first_direction, DEFAULT_FIRST_DIRECTION),
        one(initial_normal, DEFAULT_INITIAL_NORMAL),
    )


def nerf64_sincos(lengths, sin_t, cos_t, sin_p, cos_p, l0, l1, a0, p0, first_direction, initial_normal):
    """The block forward (block.cu:157-204) in sequential order, from precomputed sin/cos.

    ``lengths`` (B, S) are the step lengths L[k+2]; ``sin_t/cos_t`` (B, S) of A[k+1];
    ``sin_p/cos_p`` (B, S) of D[k].  P_k = L_0 ... L_k (affine.cuh:53-58) and
    x_{k+3} = p2 + F P_k.v; points 0..2 come from the first frame (block.cu:150-155).
    """
    ff = first_frame64(l0, l1, a0, p0, first_direction, initial_normal)
    b, steps = lengths.shape
    m = torch.eye(3, dtype=F64, device=lengths.device).expand(b, 3, 3)
    v = torch.zeros(b, 3, dtype=F64, device=lengths.device)
    pts = []
    frame, p2 = ff["frame"], ff["p2"]
    for k in range(steps):
        r, t = local_transform64(lengths[:, k], sin_t[:, k], cos_t[:, k], sin_p[:, k], cos_p[:, k])
        v = v + (m @ t[:, :, None])[:, :, 0]
        m = m @ r
        pts.append(p2 + (frame @ v[:, :, None])[:, :, 0])
    origin = p0.to(F64).expand(b, 3)
    head = [origin, ff["p1"], p2]
    return torch.stack(head + pts, dim=1)


def reconstruct64(lengths, angles, dihedrals, p0=None, first_direction=None, initial_normal=None):
    """cufk.reconstruct (reconstruct.py:29-81) restated in float64, on the inputs' device.

    Accepts (N-1,)/(N-2,)/(N-3,) or (B, ...) inputs of any float dtype; computes in float64 and
    returns (N, 3) or (B, N, 3) float64.  Differentiable w.r.t. lengths/angles/dihedrals.
    """
    single = lengths.dim() == 1
    if single:
        lengths, angles, dihedrals = lengths[None], angles[None], dihedrals[None]
    L = lengths.to(F64)
    A = angles.to(F64)
    D = dihedrals.to(F64)
    if L.shape[1] < 3:
        raise ValueError("point_count must be >= 4")
    p0_, fd_, nn_ = _anchors(p0, first_direction, initial_normal, L.device)
    xyz = nerf64_sincos(
        L[:, 2:],
        torch.sin(A[:, 1:]),
        torch.cos(A[:, 1:]),
        torch.sin(D),
        torch.cos(D),
        L[:, 0],
        L[:, 1],
        A[:, 0],
        p0_,
        fd_,
        nn_,
    )
    return xyz[0] if single else xyz


def reconstruct64_with_grads(lengths, angles, dihedrals, grad_xyz, p0=None, first_direction=None, initial_normal=None):
    """Forward plus autograd backward in float64: returns (xyz, dL, dA, dD)."""
    L = lengths.detach().to(F64).requires_grad_(True)
    A = angles.detach().to(F64).requires_grad_(True)
    D = dihedrals.detach().to(F64).requires_grad_(True)
    xyz = reconstruct64(L, A, D, p0, first_direction, initial_normal)
    gl, ga, gd = torch.autograd.grad(xyz, (L, A, D), grad_xyz.detach().to(F64))
    return xyz.detach(), gl, ga, gd


def reconstruct64_anchor_grads(lengths, angles, dihedrals, grad_xyz, p0, first_direction, initial_normal):
    """Gradients of <grad_xyz, xyz> with respect to the three anchors, by float64 autograd through
    the whole restated forward (first frame block.cu:113-148 and the chain block.cu:157-204).
    The reference itself rejects anchor gradients (extension_utils.cuh:81); this is the check for
    the extension that provides them.  Returns (xyz, d p0, d first_direction, d initial_normal)."""
    L, A, D = (x.detach().to(F64) for x in (lengths, angles, dihedrals))
    anchors = [x.detach().to(L.device, F64).requires_grad_(True) for x in (p0, first_direction, initial_normal)]
    xyz = nerf64_sincos(L[:, 2:], torch.sin(A[:, 1:]), torch.cos(A[:, 1:]), torch.sin(D), torch.cos(D), L[:, 0], L[:, 1], A[:, 0], *anchors)
    grads = torch.autograd.grad((xyz * grad_xyz.detach().to(F64)).sum(), anchors, allow_unused=True)
    # an anchor the frame does not use (the initial normal when it is parallel to the first
    # direction) has a zero gradient
    return (xyz.detach(), *(torch.zeros(3, dtype=F64, device=L.device) if gr is None else gr for gr in grads))


def block_backward64(lengths, angles, dihedrals, grad_xyz, p0=None, first_direction=None, initial_normal=None):
    """The reference's explicit backward formulas, restated in float64 (batched inputs only).

    Follows block.cu:230-313: prefix P_k (affine.cuh:53-58); suffix
    S_k = sum_{j>=k} (F^T g_{j+3} (x) P_j.v, F^T g_{j+3}) (affine.cuh:64-73, 79-84);
    local_transform_grads (affine.cuh:114-140); write_first_frame_param_grads (block.cu:206-228).
    Returns (dL, dA, dD) float64.
    """
    L = lengths.to(F64)
    A = angles.to(F64)
    D = dihedrals.to(F64)
    g = grad_xyz.to(F64)
    dev = g.device
    p0_, fd_, nn_ = _anchors(p0, first_direction, initial_normal, dev)
    b, npts = g.shape[0], g.shape[1]
    steps = npts - 3
    ff = first_frame64(L[:, 0], L[:, 1], A[:, 0], p0_, fd_, nn_)
    frame = ff["frame"]
    s_t, c_t = torch.sin(A[:, 1:]), torch.cos(A[:, 1:])
    s_p, c_p = torch.sin(D), torch.cos(D)
    pm = []
    pv = []
    m = torch.eye(3, dtype=F64, device=dev).expand(b, 3, 3)
    v = torch.zeros(b, 3, dtype=F64, device=dev)
    for k in range(steps):
        r, t = local_transform64(L[:, k + 2], s_t[:, k], c_t[:, k], s_p[:, k], c_p[:, k])
        v = v + (m @ t[:, :, None])[:, :, 0]
        m = m @ r
        pm.append(m)
        pv.append(v)
    dL = torch.zeros_like(L)
    dA = torch.zeros_like(A)
    dD = torch.zeros_like(D)
    sm = torch.zeros(b, 3, 3, dtype=F64, device=dev)
    sv = torch.zeros(b, 3, dtype=F64, device=dev)
    eye = torch.eye(3, dtype=F64, device=dev).expand(b, 3, 3)
    for k in range(steps - 1, -1, -1):
        tail = (frame.transpose(1, 2) @ g[:, k + 3, :, None])[:, :, 0]  # transpose_mul(frame, grad)
        sm = sm + tail[:, :, None] * pv[k][:, None, :]  # outer(tail, curr.v)
        sv = sv + tail
        prev_m = eye if k == 0 else pm[k - 1]
        curr_m, curr_v = pm[k], pv[k]
        grad_t = (prev_m.transpose(1, 2) @ sv[:, :, None])[:, :, 0]
        centered = sm - sv[:, :, None] * curr_v[:, None, :]
        grad_r = prev_m.transpose(1, 2) @ centered @ curr_m
        grad_r = grad_r.clone()
        grad_r[:, :, 0] = grad_r[:, :, 0] + L[:, k + 2, None] * grad_t
        s, c, S, C = s_t[:, k], c_t[:, k], s_p[:, k], c_p[:, k]
        zero = torch.zeros_like(s)
        direction = torch.stack([-c, s * C, s * S], -1)
        dtheta0 = torch.stack([s, c * C, c * S], -1)
        dtheta1 = torch.stack([-c, s * C, s * S], -1)
        dphi0 = torch.stack([zero, -s * S, s * C], -1)
        dphi1 = torch.stack([zero, c * S, -c * C], -1)
        dphi2 = torch.stack([zero, -C, -S], -1)
        col = [grad_r[:, :, i] for i in range(3)]
        dL[:, k + 2] = (grad_t * direction).sum(-1)
        dA[:, k + 1] = (col[0] * dtheta0).sum(-1) + (col[1] * dtheta1).sum(-1)
        dD[:, k] = (col[0] * dphi0).sum(-1) + (col[1] * dphi1).sum(-1) + (col[2] * dphi2).sum(-1)
    # write_first_frame_param_grads with suffix = S_0
    tail_v = (frame @ sv[:, :, None])[:, :, 0]
    tail_a = frame @ sm
    grad_p2 = g[:, 2] + tail_v
    dL[:, 0] = ((g[:, 1] + grad_p2) * ff["dir0"]).sum(-1)
    dL[:, 1] = (grad_p2 * ff["dir1"]).sum(-1)
    s0 = torch.sin(A[:, 0])[:, None]
    c0 = torch.cos(A[:, 0])[:, None]
    d_dir = s0 * ff["dir0"] + c0 * ff["turn0"]
    d_side = torch.linalg.cross(ff["normal"], d_dir, dim=-1)
    dA[:, 0] = (
        L[:, 1] * (grad_p2 * d_dir).sum(-1) + (tail_a[:, :, 0] * d_dir).sum(-1) + (tail_a[:, :, 1] * d_side).sum(-1)
    )
    return dL, dA, dD


# ---------------------------------------------------------------------------------------------
# torsion-only path (compile_torsion)
# ---------------------------------------------------------------------------------------------


def torsion_constants(bond_lengths, bond_angles):
    """torsion.cu:43-53 and torsion.py:81-86: lengths rounded to float, angle sin/cos in double."""
    lengths = tuple(float(torch.tensor(float(x), dtype=torch.float32).item()) for x in bond_lengths)
    sincos = tuple((math.sin(float(a)), math.cos(float(a))) for a in bond_angles)
    return lengths, sincos


def normalize_pairs64(raw):
    """torsion.cu:119-141: (s, c) * rsqrt(max(s^2 + c^2, 1e-16)); returns (S, C, n2)."""
    rs = raw[:, 0::2].to(F64)
    rc = raw[:, 1::2].to(F64)
    n2 = torch.clamp(rs * rs + rc * rc, min=NORM_EPS2_F32)
    inv = 1.0 / torch.sqrt(n2)
    return rs * inv, rc * inv, n2


def _torsion_tiles(bond_lengths, bond_angles, b, steps, device="cpu"):
    lengths, sincos = torsion_constants(bond_lengths, bond_angles)
    k = torch.arange(steps, device=device)
    # step k uses length phase (k+2)%3 and angle phase (k+1)%3 (torsion.cu:67-73, 219-236)
    L = torch.tensor(lengths, dtype=F64, device=device)[(k + 2) % 3].expand(b, steps)
    st = torch.tensor([sc[0] for sc in sincos], dtype=F64, device=device)[(k + 1) % 3].expand(b, steps)
    ct = torch.tensor([sc[1] for sc in sincos], dtype=F64, device=device)[(k + 1) % 3].expand(b, steps)
    l0 = torch.full((b,), lengths[0], dtype=F64, device=device)
    l1 = torch.full((b,), lengths[1], dtype=F64, device=device)
    a0 = torch.full((b,), float(bond_angles[0]), dtype=F64, device=device)
    return L, st, ct, l0, l1, a0, sincos


def torsion64(raw, bond_lengths, bond_angles):
    """compile_torsion(bond_lengths, bond_angles)(raw) restated (torsion.cu:254-295).

    Base frame = make_default_base_frame (torsion.cu:154-166), which equals the block first frame
    with default anchors; x1 = (len0, 0, 0) as base_p1 (torsion.cu:149-152).
    """
    b, width = raw.shape
    steps = width // 2
    S, C, _ = normalize_pairs64(raw)
    L, st, ct, l0, l1, a0, sincos = _torsion_tiles(bond_lengths, bond_angles, b, steps, raw.device)
    # make_default_base_frame uses the constant sin/cos of angle 0, not sin(a0) recomputed.
    xyz = _torsion_nerf(L, st, ct, S, C, l0, l1, sincos[0])
    return xyz


def _torsion_nerf(L, st, ct, S, C, l0, l1, sc0):
    b, steps = L.shape
    dev = L.device
    s0, c0 = sc0
    dir1 = torch.tensor([-c0, s0, 0.0], dtype=F64, device=dev)
    side = torch.tensor([-s0, -c0, 0.0], dtype=F64, device=dev)
    frame = torch.stack([dir1, side, torch.tensor([0.0, 0.0, 1.0], dtype=F64, device=dev)], -1).expand(b, 3, 3)
    p1 = torch.stack([l0, torch.zeros_like(l0), torch.zeros_like(l0)], -1)
    p2 = torch.stack([l0 - l1 * c0, l1 * s0, torch.zeros_like(l0)], -1)
    m = torch.eye(3, dtype=F64, device=dev).expand(b, 3, 3)
    v = torch.zeros(b, 3, dtype=F64, device=dev)
    pts = [torch.zeros(b, 3, dtype=F64, device=dev), p1, p2]
    for k in range(steps):
        r, t = local_transform64(L[:, k], st[:, k], ct[:, k], S[:, k], C[:, k])
        v = v + (m @ t[:, :, None])[:, :, 0]
        m = m @ r
        pts.append(p2 + (frame @ v[:, :, None])[:, :, 0])
    return torch.stack(pts, 1)


def torsion64_with_grads(raw, grad_xyz, bond_lengths, bond_angles):
    """Forward plus the reference's torsion backward (torsion.cu:173-217), in float64.

    World-space force/moment form of world_torsion_grad (torsion.cu:213-217): with F = sum_{j>=k+3} g_j
    and M = sum_{j>=k+3} x_j x g_j, d phi_k = ((x_{k+2} - x_{k+1}) / len_{(k+1)%3}) . (M - x_{k+2} x F);
    then the raw-pair chain rule d raw = d phi * (c_raw, -s_raw) / max(s^2 + c^2, 1e-16)
    (store_raw_pair_grad, torsion.cu:173-182).  For unclamped pairs this equals the derivative of
    the forward through atan2 (checked in tests/test_oracle.py).
    """
    b, width = raw.shape
    steps = width // 2
    S, C, n2 = normalize_pairs64(raw)
    L, st, ct, l0, l1, a0, sincos = _torsion_tiles(bond_lengths, bond_angles, b, steps, raw.device)
    xyz = _torsion_nerf(L, st, ct, S, C, l0, l1, sincos[0])
    g = grad_xyz.to(F64)
    lengths, _ = torsion_constants(bond_lengths, bond_angles)
    force = torch.flip(torch.cumsum(torch.flip(g, [1]), 1), [1])  # force[:, j] = sum_{i>=j} g_i
    moment = torch.flip(torch.cumsum(torch.flip(torch.linalg.cross(xyz, g, dim=-1), [1]), 1), [1])
    k = torch.arange(steps, device=raw.device)
    prev, pivot = xyz[:, k + 1], xyz[:, k + 2]
    Fk, Mk = force[:, k + 3], moment[:, k + 3]
    inv_len = 1.0 / torch.tensor(lengths, dtype=F64, device=raw.device)[(k + 1) % 3]
    tau = Mk - torch.linalg.cross(pivot, Fk, dim=-1)
    dphi = inv_len * ((pivot - prev) * tau).sum(-1)
    rs = raw[:, 0::2].to(F64)
    rc = raw[:, 1::2].to(F64)
    grad = torch.empty(b, width, dtype=F64, device=raw.device)
    grad[:, 0::2] = dphi * rc / n2
    grad[:, 1::2] = -dphi * rs / n2
    return xyz, grad


# ---------------------------------------------------------------------------------------------
# synthetic inputs shared by tests and the benchmark (no public dataset exists for this path)
# ---------------------------------------------------------------------------------------------

BACKBONE_LENGTHS = (0.14685231, 0.15365194, 0.13405086)
BACKBONE_ANGLES = (1.9676635, 2.062335, 2.164016)


def make_inputs(batch: int, points: int, seed: int = 0, dtype=torch.float32, anchors: bool = False):
    """Seeded synthetic backbone internal coordinates, generated in float64 on the CPU then cast.

    lengths cycle the backbone bond lengths + N(0, 0.002); angles cycle the backbone bond angles
    + N(0, 0.03); dihedrals ~ U(-pi, pi); grad_out ~ N(0, 1).  With ``anchors`` p0 ~ N(0, 1)^3 and
    first_direction / initial_normal are a random orthonormal pair.
    """
    g = torch.Generator().manual_seed(seed)
    i1 = torch.arange(points - 1)
    i2 = torch.arange(points - 2)
    L = torch.tensor(BACKBONE_LENGTHS, dtype=F64)[i1 % 3] + 0.002 * torch.randn(batch, points - 1, generator=g, dtype=F64)
    A = torch.tensor(BACKBONE_ANGLES, dtype=F64)[i2 % 3] + 0.03 * torch.randn(batch, points - 2, generator=g, dtype=F64)
    D = (torch.rand(batch, points - 3, generator=g, dtype=F64) * 2.0 - 1.0) * math.pi
    G = torch.randn(batch, points, 3, generator=g, dtype=F64)
    out = {"lengths": L.to(dtype), "angles": A.to(dtype), "dihedrals": D.to(dtype), "grad": G.to(dtype)}
    if anchors:
        p0 = torch.randn(3, generator=g, dtype=F64)
        q, _ = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=F64))
        out["p0"] = p0.to(dtype)
        out["first_direction"] = q[:, 0].contiguous().to(dtype)
        out["initial_normal"] = q[:, 1].contiguous().to(dtype)
    return out


def make_torsion_inputs(batch: int, points: int, seed: int = 0, dtype=torch.float32):
    """raw (B, 2(N-3)) ~ N(0, 1) interleaved [sin, cos]; grad_out (B, N, 3) ~ N(0, 1)."""
    g = torch.Generator().manual_seed(seed)
    raw = torch.randn(batch, 2 * (points - 3), generator=g, dtype=F64)
    G = torch.randn(batch, points, 3, generator=g, dtype=F64)
    return {"raw": raw.to(dtype), "grad": G.to(dtype)}
