"""Chunked gated delta rule: forward and hand-derived backward.

Per chunk of C tokens with incoming state S0 (dk x dv), cumulative log decay gamma_t
within the chunk (Gamma = diag(exp(gamma))), q already L2-normalised and scaled, k
L2-normalised:

    E_ts = exp(gamma_t - gamma_s)
    A    = strictly_lower(diag(beta) (E * K K^T))
    U    = (I + A)^{-1} diag(beta) (V - Gamma K S0)          (forward substitution)
    O    = Gamma Q S0 + lower_incl(E * Q K^T) U
    S_C  = exp(gamma_C) S0 + K^T diag(exp(gamma_C - gamma)) U

which equals the token recurrence S_t = e^{g_t} S_{t-1} + k_t u_t^T,
u_t = beta_t (v_t - e^{g_t} S_{t-1}^T k_t), o_t = S_t^T q_t.  The backward walks the chunks
in reverse carrying dS and differentiates those five lines (see ``chunk_bwd``); the states
at chunk starts are saved by the forward.

This module is the statement the CUDA kernels in ``csrc/gdn.cu`` implement (same
chunking, same order of operations) and their oracle; it also runs on CPU.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _chunks(t_len: int, c: int):
    return [(s, min(t_len, s + c)) for s in range(0, t_len, c)]


def chunk_fwd(q, k, v, g, beta, s0=None, chunk: int = 64, per_channel: bool = False):
    """One sequence, one head: q/k (T, dk) (already normalised/scaled), v (T, dv), g (T,) or
    (T, dk) log decay, beta (T,).  Returns (o (T, dv), final state, chunk start states)."""
    t_len, dk = k.shape
    dv = v.shape[-1]
    dt = torch.promote_types(q.dtype, torch.float32)
    s = torch.zeros(dk, dv, dtype=dt, device=q.device) if s0 is None else s0.to(dt).clone()
    out = torch.zeros(t_len, dv, dtype=dt, device=q.device)
    states = []
    for a, b in _chunks(t_len, chunk):
        states.append(s.clone())
        Q, K, V, B = q[a:b].to(dt), k[a:b].to(dt), v[a:b].to(dt), beta[a:b].to(dt)
        gam = torch.cumsum(g[a:b].to(dt), 0)  # (C,) or (C, dk)
        if per_channel:
            # E_ts per channel: apply the decay to k / q along dk
            Kd = K * torch.exp(gam)              # k_t scaled by decay to t (for Gamma K S0)
            Kinv = K * torch.exp(-gam)           # k_s / decay(s)
            Qd = Q * torch.exp(gam)
            A = torch.tril(B[:, None] * (Kd @ Kinv.t()), -1)
            W = V - Kd @ s
            U = torch.linalg.solve_triangular(torch.eye(b - a, device=q.device, dtype=dt) + A, B[:, None] * W,
                                              upper=False, unitriangular=True)
            P = torch.tril(Qd @ Kinv.t())
            out[a:b] = Qd @ s + P @ U
            gl = gam[-1]
            s = torch.exp(gl)[:, None] * s + (K * torch.exp(gl[None, :] - gam)).t() @ U
        else:
            E = torch.exp(gam[:, None] - gam[None, :])
            A = torch.tril(B[:, None] * E * (K @ K.t()), -1)
            W = V - torch.exp(gam)[:, None] * (K @ s)
            U = torch.linalg.solve_triangular(torch.eye(b - a, device=q.device, dtype=dt) + A, B[:, None] * W,
                                              upper=False, unitriangular=True)
            P = torch.tril(E * (Q @ K.t()))
            out[a:b] = torch.exp(gam)[:, None] * (Q @ s) + P @ U
            gl = gam[-1]
            s = torch.exp(gl) * s + (K * torch.exp(gl - gam)[:, None]).t() @ U
    return out, s, states


def chunk_fwd_batched(q, k, v, g, beta, s0=None, chunk: int = 64, per_channel: bool = False):
    """``chunk_fwd`` over a batch of independent (sequence, head) rows at once: q/k (N, T, dk)
    (already normalised / scaled), v (N, T, dv), g (N, T) or (N, T, dk), beta (N, T), s0
    (N, dk, dv) or None.  Rows shorter than T are padded at the end with zeros (zero k, v,
    beta and g leave the state unchanged).  Returns (o (N, T, dv), final states (N, dk, dv));
    differentiable, so autograd gives the backward.  Only the walk over chunks is a Python
    loop: every product is one batched matmul / triangular solve over the N rows."""
    n, t_len, dk = k.shape
    dv = v.shape[-1]
    dt = torch.promote_types(q.dtype, torch.float32)
    s = torch.zeros(n, dk, dv, dtype=dt, device=q.device) if s0 is None else s0.to(dt)
    outs = []
    for a, b in _chunks(t_len, chunk):
        Q, K, V, B = q[:, a:b].to(dt), k[:, a:b].to(dt), v[:, a:b].to(dt), beta[:, a:b].to(dt)
        gam = torch.cumsum(g[:, a:b].to(dt), 1)  # (n, c) or (n, c, dk)
        eye = torch.eye(b - a, device=q.device, dtype=dt)
        if per_channel:
            up, down = torch.exp(gam), torch.exp(-gam)
            Kd, Kinv, Qd = K * up, K * down, Q * up
            A = torch.tril(B[..., None] * (Kd @ Kinv.transpose(1, 2)), -1)
            W = V - Kd @ s
            P = torch.tril(Qd @ Kinv.transpose(1, 2))
            U = torch.linalg.solve_triangular(eye + A, B[..., None] * W, upper=False, unitriangular=True)
            outs.append(Qd @ s + P @ U)
            gl = gam[:, -1]  # (n, dk)
            s = torch.exp(gl)[..., None] * s + (K * torch.exp(gl[:, None, :] - gam)).transpose(1, 2) @ U
        else:
            E = torch.exp(gam[:, :, None] - gam[:, None, :])
            eg = torch.exp(gam)[..., None]
            A = torch.tril(B[..., None] * E * (K @ K.transpose(1, 2)), -1)
            W = V - eg * (K @ s)
            P = torch.tril(E * (Q @ K.transpose(1, 2)))
            U = torch.linalg.solve_triangular(eye + A, B[..., None] * W, upper=False, unitriangular=True)
            outs.append(eg * (Q @ s) + P @ U)
            gl = gam[:, -1]  # (n,)
            s = torch.exp(gl)[:, None, None] * s + (K * torch.exp(gl[:, None] - gam)[..., None]).transpose(1, 2) @ U
    return torch.cat(outs, 1), s


def chunk_bwd(q, k, v, g, beta, states, do, ds_final=None, chunk: int = 64):
    """Gradients (dq, dk, dv, dg, dbeta, ds0) of chunk_fwd (scalar decay per head)."""
    t_len, dk = k.shape
    dv_dim = v.shape[-1]
    dt = torch.promote_types(q.dtype, torch.float32)
    dq = torch.zeros(q.shape, dtype=dt, device=q.device)
    dk_ = torch.zeros(k.shape, dtype=dt, device=q.device)
    dv = torch.zeros(v.shape, dtype=dt, device=q.device)
    dg = torch.zeros(t_len, dtype=dt, device=q.device)
    db = torch.zeros(t_len, dtype=dt, device=q.device)
    dS = torch.zeros(dk, dv_dim, dtype=dt, device=q.device) if ds_final is None else ds_final.to(dt).clone()
    spans = _chunks(t_len, chunk)
    for ci in range(len(spans) - 1, -1, -1):
        a, b = spans[ci]
        s0 = states[ci].to(dt)
        Q, K, V, B = q[a:b].to(dt), k[a:b].to(dt), v[a:b].to(dt), beta[a:b].to(dt)
        dO = do[a:b].to(dt)
        c = b - a
        gam = torch.cumsum(g[a:b].to(dt), 0)
        eg = torch.exp(gam)
        E = torch.exp(gam[:, None] - gam[None, :])
        KK = K @ K.t()
        A = torch.tril(B[:, None] * E * KK, -1)
        KS = K @ s0
        R = V - eg[:, None] * KS
        Y = B[:, None] * R
        I = torch.eye(c, device=q.device, dtype=dt)
        U = torch.linalg.solve_triangular(I + A, Y, upper=False, unitriangular=True)
        QK = Q @ K.t()
        P = torch.tril(E * QK)
        gl = gam[-1]
        Fw = torch.exp(gl - gam)
        # dU from O = Gamma Q S0 + P U and S_C = e^{gl} S0 + K^T F U
        dU = P.t() @ dO + Fw[:, None] * (K @ dS)
        dP = torch.tril(dO @ U.t())
        # U = (I + A)^{-1} Y
        dY = torch.linalg.solve_triangular((I + A).t(), dU, upper=True, unitriangular=True)
        dA = torch.tril(-dY @ U.t(), -1)
        dR = B[:, None] * dY
        dbeta = (dY * R).sum(1)
        dV = dR
        # R = V - Gamma K S0
        dKS = -eg[:, None] * dR
        dgam = -(eg[:, None] * KS * dR).sum(1)
        dK = dKS @ s0.t()
        dS0 = K.t() @ dKS
        # A = tril(diag(B) E KK, -1)
        dAE = dA * E
        dbeta = dbeta + (dAE * KK).sum(1)
        dKK = dAE * B[:, None]
        dK = dK + dKK @ K + dKK.t() @ K
        dEA = dA * B[:, None] * KK * E
        dgam = dgam + dEA.sum(1) - dEA.sum(0)
        # P = tril(E QK)
        dPE = dP * E
        dQ = dPE @ K
        dK = dK + dPE.t() @ Q
        dEP = dP * P
        dgam = dgam + dEP.sum(1) - dEP.sum(0)
        # Gamma Q S0
        QS = Q @ s0
        dQ = dQ + eg[:, None] * (dO @ s0.t())
        dgam = dgam + eg * (QS * dO).sum(1)
        dS0 = dS0 + Q.t() @ (eg[:, None] * dO)
        # S_C = e^{gl} S0 + K^T F U
        dS0 = dS0 + torch.exp(gl) * dS
        dFw = ((K @ dS) * U).sum(1)
        dK = dK + Fw[:, None] * (U @ dS.t())
        dgl = torch.exp(gl) * (s0 * dS).sum() + (dFw * Fw).sum()
        dgam = dgam - dFw * Fw
        dgam[-1] = dgam[-1] + dgl
        dq[a:b], dk_[a:b], dv[a:b], db[a:b] = dQ, dK, dV, dbeta
        dg[a:b] = torch.flip(torch.cumsum(torch.flip(dgam, [0]), 0), [0])
        dS = dS0
    return dq, dk_, dv, dg, db, dS


def l2norm_bwd(x: torch.Tensor, dy: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Gradient of F.normalize(x, dim=-1, eps) given the output gradient."""
    xf = x.float()
    n = xf.norm(dim=-1, keepdim=True).clamp(min=eps)
    y = xf / n
    return (dy - y * (y * dy).sum(-1, keepdim=True)) / n
