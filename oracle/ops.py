"""PyTorch CPU restatement of the reference ops (test infrastructure, see ``oracle/__init__``).

Every function follows the reference op of the same name; the file:line it
restates is in its docstring. Forward passes are written with differentiable
torch ops, so ``torch.autograd`` supplies the backward the reference's
hand-written kernels compute (up to O(1e-7) terms the reference drops, e.g. the
eps inside its normalisations). Arithmetic is fp32 like the reference, except
where the reference accumulates in fp64 (the two CSR scatters), which is kept.
Passing fp64 tensors gives an fp64 oracle.

Wigner-D layout ([E, 34], ``ops/constants.py:6-16``): D1 row-major 3x3 in
columns 0-8, D2 row-major 5x5 in columns 9-33. D1 is the rotation matrix of the
edge-frame quaternion (it maps the edge direction onto +y). D2 is computed here
as the l=2 representation of that rotation in the real basis
(xz, xy, (2y^2-x^2-z^2)/sqrt6, yz, (z^2-x^2)/sqrt2) of symmetric traceless
matrices, D2[a,b] = tr(R^T B_a R B_b); the reference expands the same matrix as
quartic polynomials of the quaternion (``ops/geom.py:141-178``). The golden
vectors pin the two to ~1e-6.
"""
from __future__ import annotations

import math

import torch

SQRT2_INV = 1.0 / math.sqrt(2.0)
SQRT6_INV = 1.0 / math.sqrt(6.0)


def l2_basis(dtype=torch.float64) -> torch.Tensor:
    """The 5 symmetric traceless 3x3 matrices B_a (Frobenius-orthonormal), [5, 3, 3]."""
    B = torch.zeros(5, 3, 3, dtype=dtype)
    B[0, 0, 2] = B[0, 2, 0] = SQRT2_INV          # xz
    B[1, 0, 1] = B[1, 1, 0] = SQRT2_INV          # xy
    B[2, 0, 0] = -SQRT6_INV; B[2, 1, 1] = 2 * SQRT6_INV; B[2, 2, 2] = -SQRT6_INV  # polar (y)
    B[3, 1, 2] = B[3, 2, 1] = SQRT2_INV          # yz
    B[4, 0, 0] = -SQRT2_INV; B[4, 2, 2] = SQRT2_INV  # z^2 - x^2
    return B


def quat_to_rotation(qw, qx, qy, qz):
    """Standard quaternion -> rotation matrix, [E, 3, 3] (``ops/geom.py:133-139``)."""
    xx, yy, zz = qx * qx, qy * qy, qz * qz
    xy, xz, yz = qx * qy, qx * qz, qy * qz
    wx, wy, wz = qw * qx, qw * qy, qw * qz
    r0 = torch.stack([1 - 2 * (yy + zz), 2 * (xy - wz), 2 * (xz + wy)], -1)
    r1 = torch.stack([2 * (xy + wz), 1 - 2 * (xx + zz), 2 * (yz - wx)], -1)
    r2 = torch.stack([2 * (xz - wy), 2 * (yz + wx), 1 - 2 * (xx + yy)], -1)
    return torch.stack([r0, r1, r2], -2)


def wigner_l2(R: torch.Tensor) -> torch.Tensor:
    """D2[a, b] = tr(R^T B_a R B_b) for R [E, 3, 3] -> [E, 5, 5]."""
    B = l2_basis(R.dtype)
    M = torch.einsum("eki,akl,elj->eaij", R, B, R)  # R^T B_a R
    return torch.einsum("eaij,bij->eab", M, B)


def edge_frame_quaternion(ex, ey, ez, eps: float = 1e-7):
    """Two-chart edge-frame quaternion (``ops/geom.py:106-131``).

    Chart 1 rotates the unit edge vector e onto +y through the half-way
    quaternion (1+e_y, -e_z, 0, e_x); chart 2 is (-e_z, 1-e_y, e_x, 0), regular
    where chart 1 degenerates (e_y -> -1). They are blended with
    s = sigmoid((2t-1)/max(t(1-t), eps)), t = clamp((e_y+0.9)/1.8, 0, 1), s
    forced to 0 / 1 at the ends, after flipping chart 1 onto chart 2's
    hemisphere; the blend is renormalised with eps inside the root."""
    n1 = torch.sqrt((1.0 + ey) ** 2 + ez * ez + ex * ex + eps)
    q1w, q1x, q1z = (1.0 + ey) / n1, -ez / n1, ex / n1
    n2 = torch.sqrt(ez * ez + (1.0 - ey) ** 2 + ex * ex + eps)
    q2w, q2x, q2y = -ez / n2, (1.0 - ey) / n2, ex / n2
    t = torch.clamp((ey + 0.9) / 1.8, 0.0, 1.0)
    num = 2.0 * t - 1.0
    den = torch.clamp(t * (1.0 - t), min=eps)
    s = torch.sigmoid(num / den)
    s = torch.where(t < eps, torch.zeros_like(s), s)
    s = torch.where(t > 1.0 - eps, torch.ones_like(s), s)
    flip = (q1w * q2w + q1x * q2x) < 0.0
    sign = torch.where(flip, -torch.ones_like(q1w), torch.ones_like(q1w))
    q1w, q1x, q1z = q1w * sign, q1x * sign, q1z * sign
    qw = (1.0 - s) * q2w + s * q1w
    qx = (1.0 - s) * q2x + s * q1x
    qy = (1.0 - s) * q2y
    qz = s * q1z
    ne = torch.sqrt(qw * qw + qx * qx + qy * qy + qz * qz + eps)
    return qw / ne, qx / ne, qy / ne, qz / ne


def envelope(dist: torch.Tensor, cutoff: float) -> torch.Tensor:
    """Polynomial envelope 1 - 21u^5 + 35u^6 - 15u^7, zero for u >= 1 (``ops/geom.py:78-82``)."""
    u = dist / cutoff
    u5 = (u * u) * (u * u) * u
    env = 1.0 + u5 * (-21.0 + u * (35.0 - 15.0 * u))
    return torch.where(u < 1.0, env, torch.zeros_like(env))


def precompute_geometry(pos, Z, idx_i, idx_j, shifts, W_src, W_tgt, offset_g, coeff_g, cutoff):
    """Restates ``ops/geom.py:36-214`` (forward) + ``:496-531``.

    Returns x_edge_raw [E, B+2C] = [gaussians, W_src[Z_i], W_tgt[Z_j]], wigner [E, 34], env [E]."""
    d = pos[idx_i] - pos[idx_j] + shifts
    dist = torch.sqrt((d * d).sum(-1))
    dist_safe = torch.clamp(dist, min=1e-7)
    env = envelope(dist, cutoff)
    gauss = torch.exp(coeff_g * (dist[:, None] - offset_g[None, :]) ** 2)
    x_edge = torch.cat([gauss, W_src[Z[idx_i]].to(gauss.dtype), W_tgt[Z[idx_j]].to(gauss.dtype)], dim=1)
    e = d / dist_safe[:, None]
    qw, qx, qy, qz = edge_frame_quaternion(e[:, 0], e[:, 1], e[:, 2])
    R = quat_to_rotation(qw, qx, qy, qz)
    D2 = wigner_l2(R)
    wigner = torch.cat([R.reshape(-1, 9), D2.reshape(-1, 25)], dim=1)
    return x_edge, wigner, env


def layer_norm_silu(x, gamma, beta, eps: float = 1e-7):
    """Row-wise LayerNorm (biased variance, eps 1e-7) then SiLU (``ops/ln_silu.py:29-72,180-185``)."""
    mean = x.mean(dim=1, keepdim=True)
    xc = x - mean
    var = (xc * xc).mean(dim=1, keepdim=True)
    y = xc * torch.rsqrt(var + eps) * gamma + beta
    return y * torch.sigmoid(y)


def _split_rows(wigner):
    D1 = wigner[:, :9].reshape(-1, 3, 3)
    D2 = wigner[:, 9:].reshape(-1, 5, 5)
    return D1, D2


def gather_wigner_split(x_in, idx_i, idx_j, wigner, rad_out, csd_emb, batch):
    """Restates ``ops/gather.py:34-154`` (+ ``:408-433``).

    For edge e = (i -> j): v = x[i] / x[j] with the system embedding added to l=0,
    rotated into the edge frame (D1 on l=1, D2 on l=2), each rotated coefficient
    scaled by its radial slot. Output layout per edge, C channels per slot:
    X_m0 = [v_i0 r0, v_j0 r1, (D1 v_i)_1 r2, (D1 v_j)_1 r3, (D2 v_i)_2 r4, (D2 v_j)_2 r5]
    X_m1 = [(D1 v_i)_2 r6, (D1 v_j)_2 r7, (D2 v_i)_3 r8, (D2 v_j)_3 r9,
            (D1 v_i)_0 r6, (D1 v_j)_0 r7, (D2 v_i)_1 r8, (D2 v_j)_1 r9]
    X_m2 = [(D2 v_i)_4 r10, (D2 v_j)_4 r11, (D2 v_i)_0 r10, (D2 v_j)_0 r11]
    (0-based rotated-row indices; D1 row 1 / D2 row 2 are m=0)."""
    C = x_in.shape[2]
    D1, D2 = _split_rows(wigner)
    ce = csd_emb[batch]
    vi = x_in[idx_i].clone(); vj = x_in[idx_j].clone()
    vi = torch.cat([vi[:, :1] + ce[idx_i][:, None], vi[:, 1:]], dim=1)
    vj = torch.cat([vj[:, :1] + ce[idx_j][:, None], vj[:, 1:]], dim=1)
    ri1 = torch.einsum("erk,ekc->erc", D1, vi[:, 1:4]); rj1 = torch.einsum("erk,ekc->erc", D1, vj[:, 1:4])
    ri2 = torch.einsum("erk,ekc->erc", D2, vi[:, 4:9]); rj2 = torch.einsum("erk,ekc->erc", D2, vj[:, 4:9])
    r = rad_out.reshape(-1, 12, C)
    X_m0 = torch.stack([vi[:, 0] * r[:, 0], vj[:, 0] * r[:, 1], ri1[:, 1] * r[:, 2], rj1[:, 1] * r[:, 3],
                        ri2[:, 2] * r[:, 4], rj2[:, 2] * r[:, 5]], 1)
    X_m1 = torch.stack([ri1[:, 2] * r[:, 6], rj1[:, 2] * r[:, 7], ri2[:, 3] * r[:, 8], rj2[:, 3] * r[:, 9],
                        ri1[:, 0] * r[:, 6], rj1[:, 0] * r[:, 7], ri2[:, 1] * r[:, 8], rj2[:, 1] * r[:, 9]], 1)
    X_m2 = torch.stack([ri2[:, 4] * r[:, 10], rj2[:, 4] * r[:, 11], ri2[:, 0] * r[:, 10], rj2[:, 0] * r[:, 11]], 1)
    return X_m0.reshape(-1, 6 * C), X_m1.reshape(-1, 8 * C), X_m2.reshape(-1, 4 * C)


def fused_gating_split(Y_m0, Y_m1, Y_m2, C):
    """Restates ``ops/gating.py:32-103``: g0 = sigmoid(Y0[0]), g1 = sigmoid(Y0[1]);
    Z_m0 = [silu(Y0[2]), Y0[3] g0, Y0[4] g1]; Z_m1 = [Y1[0] g0, Y1[1] g1, Y1[2] g0, Y1[3] g1];
    Z_m2 = [Y2[0] g1, Y2[1] g1] (C-wide slots)."""
    y0 = Y_m0.reshape(-1, 5, C); y1 = Y_m1.reshape(-1, 4, C); y2 = Y_m2.reshape(-1, 2, C)
    g0 = torch.sigmoid(y0[:, 0]); g1 = torch.sigmoid(y0[:, 1])
    Z0 = torch.stack([y0[:, 2] * torch.sigmoid(y0[:, 2]), y0[:, 3] * g0, y0[:, 4] * g1], 1)
    Z1 = torch.stack([y1[:, 0] * g0, y1[:, 1] * g1, y1[:, 2] * g0, y1[:, 3] * g1], 1)
    Z2 = torch.stack([y2[:, 0] * g1, y2[:, 1] * g1], 1)
    return Z0.reshape(-1, 3 * C), Z1.reshape(-1, 4 * C), Z2.reshape(-1, 2 * C)


def _rotate_back(Z_m0, Z_m1, Z_m2, wigner, C):
    """Per-edge M->L inverse rotation (``ops/scatter.py:117-127``): out [E, 9, C] with
    l0 = Z0[0]; l1 = D1^T (Z1[2], Z0[1], Z1[0]); l2 = D2^T (Z2[1], Z1[3], Z0[2], Z1[1], Z2[0])."""
    D1, D2 = _split_rows(wigner)
    z0 = Z_m0.reshape(-1, 3, C); z1 = Z_m1.reshape(-1, 4, C); z2 = Z_m2.reshape(-1, 2, C)
    m1 = torch.stack([z1[:, 2], z0[:, 1], z1[:, 0]], 1)               # rows of the l=1 edge frame
    m2 = torch.stack([z2[:, 1], z1[:, 3], z0[:, 2], z1[:, 1], z2[:, 0]], 1)
    l1 = torch.einsum("erk,erc->ekc", D1, m1)
    l2 = torch.einsum("erk,erc->ekc", D2, m2)
    return torch.cat([z0[:, :1], l1, l2], dim=1)


def rotate_scatter_split(Z_m0, Z_m1, Z_m2, wigner, env, x_res, idx_j, row_ptr, col_idx, N):
    """Restates ``ops/scatter.py:45-140`` (+ ``:295-315``): x_out[j] = x_res[j] + sum over
    edges e with destination j of env_e * rotate_back(Z_e), products in the input
    precision, sum in fp64, result cast back. The sum runs over ``idx_j`` (the CSR
    only fixes the order, which fp64 makes immaterial at fp32 output precision)."""
    C = x_res.shape[2]
    contrib = _rotate_back(Z_m0, Z_m1, Z_m2, wigner, C) * env[:, None, None]
    acc = torch.zeros(N, 9, C, dtype=torch.float64).index_add(0, idx_j, contrib.to(torch.float64))
    return (acc + x_res.to(torch.float64)).to(x_res.dtype)


def init_node_scatter(rad_out, wigner, env, Z, batch, W_sphere, csd_emb, idx_j, row_ptr, col_idx, N):
    """Restates ``ops/scatter.py:360-423`` (+ ``:484-501``): initial node embedding
    x[n] = W_sphere[Z_n] + csd[batch_n] (l=0) + sum over edges into n of env/5 times
    [r0, r1 * D1[1, :], r2 * D2[2, :]] (the m=0 rows), fp64 sum."""
    C = rad_out.shape[1] // 3
    D1, D2 = _split_rows(wigner)
    r = rad_out.reshape(-1, 3, C)
    envc = env[:, None]
    l0 = (r[:, 0] * envc) / 5.0
    l1 = (r[:, 1][:, None, :] * D1[:, 1, :, None] * envc[:, None]) / 5.0
    l2 = (r[:, 2][:, None, :] * D2[:, 2, :, None] * envc[:, None]) / 5.0
    contrib = torch.cat([l0[:, None], l1, l2], dim=1)
    acc = torch.zeros(N, 9, C, dtype=torch.float64).index_add(0, idx_j, contrib.to(torch.float64))
    base = torch.zeros(N, 9, C, dtype=torch.float64)
    base[:, 0] = (W_sphere[Z] + csd_emb[batch]).to(torch.float64)
    return (base + acc).to(rad_out.dtype)
