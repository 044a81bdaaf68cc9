"""Chunked KDA in plain PyTorch, stage by stage (TEST INFRASTRUCTURE ONLY).

The CUDA path splits the layer into stages; this file computes the same
stages with the same algebra in float64 so that the GPU tests can compare
intermediate tensors, and so that the hand-derived backward is checked against
autograd of the per-token oracle.  Notation (per sequence, per head, chunk of
C=64 tokens, D=128):

  Gam   = inclusive cumsum of the log decay g inside the chunk
  L'    = strictly lower  [k_i . (k_j * exp(Gam_i - Gam_j))]
  M     = lower incl diag [q_i . (k_j * exp(Gam_i - Gam_j))]        (Aqk)
  A     = (I + diag(beta) L')^-1,  T = A diag(beta)
  W     = T (k * exp(Gam)),  U = T v
  Qt    = q * exp(Gam),  Kb = k * exp(Gam_C - Gam),  dC = exp(Gam_C)
  E     = U - W S0,  O = Qt S0 + M E,  S_C = diag(dC) S0 + Kb^T E

Backward per chunk given dO and dS_C (gradient of the chunk-end state):

  dE = M^T dO + Kb dS_C;  dS0 = Qt^T dO + diag(dC) dS_C - W^T dE
  then the chunk-local gradients of ``chunk_backward``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

C = 64


def prologue(q_in, k_in, v_in, g_logits, beta_logits, A_log, dt_bias, lower_bound, scale):
    """[B,T,H,D] post-conv inputs -> normalised q (scaled), k, v, g, beta and
    the saved norms."""
    H, D = q_in.shape[-2:]
    qn = q_in.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    kn = k_in.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    z = torch.exp(A_log).view(1, 1, H, 1) * (g_logits + dt_bias.view(1, 1, H, D))
    g = lower_bound * torch.sigmoid(z)
    beta = torch.sigmoid(beta_logits)
    return q_in / qn * scale, k_in / kn, v_in, g, beta, qn, kn, z


def _to_chunks(x, T):
    """[B,T,H,...] -> [B,H,NT,C,...] zero padded."""
    NT = (T + C - 1) // C
    pad = NT * C - T
    if pad:
        x = F.pad(x, [0, 0] * (x.dim() - 2) + [0, pad]) if x.dim() > 3 else F.pad(x, (0, 0, 0, pad))
    B, H = x.shape[0], x.shape[2]
    x = x.reshape(B, NT, C, H, *x.shape[3:])
    return x.movedim(3, 1)


def _from_chunks(x, T):
    B, H, NT = x.shape[:3]
    x = x.movedim(1, 3).reshape(B, NT * C, H, *x.shape[4:])
    return x[:, :T]


def intra(q, k, v, g, beta):
    """Chunk-parallel stage.  Inputs [B,H,NT,C,D] (beta [B,H,NT,C])."""
    Gam = g.cumsum(-2)
    diff = Gam.unsqueeze(-2) - Gam.unsqueeze(-3)             # [.., i, j, D]
    tri_strict = torch.tril(torch.ones(C, C, dtype=torch.bool), -1)
    tri_incl = torch.tril(torch.ones(C, C, dtype=torch.bool), 0)
    ex = torch.exp(torch.where(tri_incl[..., None], diff, torch.zeros_like(diff)))
    Lp = torch.einsum("...id,...jd,...ijd->...ij", k, k, ex).masked_fill(~tri_strict, 0)
    M = torch.einsum("...id,...jd,...ijd->...ij", q, k, ex).masked_fill(~tri_incl, 0)
    eye = torch.eye(C, dtype=q.dtype)
    A = torch.linalg.inv(eye + beta.unsqueeze(-1) * Lp)
    Tm = A * beta.unsqueeze(-2)
    eG = torch.exp(Gam)
    GC = Gam[..., -1:, :]
    W = Tm @ (k * eG)
    U = Tm @ v
    Qt = q * eG
    Kb = k * torch.exp(GC - Gam)
    dC = torch.exp(GC[..., 0, :])
    return dict(Gam=Gam, Lp=Lp, M=M, A=A, Tm=Tm, W=W, U=U, Qt=Qt, Kb=Kb, dC=dC)


def state_forward(it, S0):
    """Sequential stage.  S0 [B,H,D,D].  Returns O, h (chunk-start states), E, S_T."""
    NT = it["W"].shape[2]
    S = S0
    O, hs, Es = [], [], []
    for n in range(NT):
        hs.append(S)
        E = it["U"][:, :, n] - it["W"][:, :, n] @ S
        O.append(it["Qt"][:, :, n] @ S + it["M"][:, :, n] @ E)
        S = it["dC"][:, :, n].unsqueeze(-1) * S + it["Kb"][:, :, n].transpose(-1, -2) @ E
        Es.append(E)
    return torch.stack(O, 2), torch.stack(hs, 2), torch.stack(Es, 2), S


def state_backward(it, dO, dST):
    """Reverse sequential stage.  Returns dE, dh (chunk-end state grads), dS0."""
    NT = it["W"].shape[2]
    dS = dST
    dEs, dhs = [None] * NT, [None] * NT
    for n in reversed(range(NT)):
        dE = it["M"][:, :, n].transpose(-1, -2) @ dO[:, :, n] + it["Kb"][:, :, n] @ dS
        dhs[n] = dS
        dS = (it["Qt"][:, :, n].transpose(-1, -2) @ dO[:, :, n]
              + it["dC"][:, :, n].unsqueeze(-1) * dS - it["W"][:, :, n].transpose(-1, -2) @ dE)
        dEs[n] = dE
    return torch.stack(dEs, 2), torch.stack(dhs, 2), dS


def chunk_backward(q, k, v, g, beta, it, h, dh, E, dE, dO):
    """Chunk-parallel backward: returns dq, dk, dv (of normalised/scaled inputs),
    dg (log decay, before the gate), dbeta (sigmoid output)."""
    Gam, A, Tm, Lp = it["Gam"], it["A"], it["Tm"], it["Lp"]
    eG = torch.exp(Gam)
    GC = Gam[..., -1:, :]
    eGC = torch.exp(GC - Gam)
    tri_strict = torch.tril(torch.ones(C, C, dtype=torch.bool), -1)
    tri_incl = torch.tril(torch.ones(C, C, dtype=torch.bool), 0)
    S0, dSC = h, dh
    dQt = dO @ S0.transpose(-1, -2)
    dM = (dO @ E.transpose(-1, -2)).masked_fill(~tri_incl, 0)
    dKb = E @ dSC.transpose(-1, -2)
    dDC = (dSC * S0).sum(-1)
    dW = -dE @ S0.transpose(-1, -2)
    dU = dE
    dv = Tm.transpose(-1, -2) @ dU
    Ke = k * eG
    dKe = Tm.transpose(-1, -2) @ dW
    dT = dU @ v.transpose(-1, -2) + dW @ Ke.transpose(-1, -2)
    dbeta = (dT * A).sum(-2)
    dA = dT * beta.unsqueeze(-2)
    dL = -(A.transpose(-1, -2) @ dA @ A.transpose(-1, -2))
    dL = dL.masked_fill(~tri_strict, 0)
    dbeta = dbeta + (dL * Lp).sum(-1)
    dLp = dL * beta.unsqueeze(-1)
    diff = Gam.unsqueeze(-2) - Gam.unsqueeze(-3)
    ex = torch.exp(torch.where(tri_incl[..., None], diff, torch.zeros_like(diff)))
    dq_M = torch.einsum("...ij,...jd,...ijd->...id", dM, k, ex)
    dk_M = torch.einsum("...ij,...id,...ijd->...jd", dM, q, ex)
    dk_Lr = torch.einsum("...ij,...jd,...ijd->...id", dLp, k, ex)
    dk_Lc = torch.einsum("...ij,...id,...ijd->...jd", dLp, k, ex)
    dq = dQt * eG + dq_M
    dk = dKe * eG + dKb * eGC + dk_M + dk_Lr + dk_Lc
    dGam = (q * dQt * eG + Ke * dKe - k * eGC * dKb + q * dq_M - k * dk_M
            + k * dk_Lr - k * dk_Lc)
    last = (k * eGC * dKb).sum(-2) + it["dC"] * dDC
    dGam[..., -1, :] = dGam[..., -1, :] + last
    dg = dGam.flip(-2).cumsum(-2).flip(-2)
    return dq, dk, dv, dg, dbeta


def prologue_backward(q_in, k_in, qn, kn, z, beta, A_log, lower_bound, scale,
                      dq, dk, dg, dbeta):
    """Chain rule through the L2 norms, the gate and the beta sigmoid."""
    nq = q_in / qn
    nk = k_in / kn
    dnq = dq * scale
    dq_in = (dnq - nq * (nq * dnq).sum(-1, keepdim=True)) / qn
    dk_in = (dk - nk * (nk * dk).sum(-1, keepdim=True)) / kn
    s = torch.sigmoid(z)
    dz = dg * lower_bound * s * (1 - s)
    H = q_in.shape[2]
    dx = dz * torch.exp(A_log).view(1, 1, H, 1)
    dA_log = (dz * z).sum(dim=(0, 1, 3))
    ddt_bias = dx.sum(dim=(0, 1)).reshape(-1)
    dbeta_logits = dbeta * beta * (1 - beta)
    return dq_in, dk_in, dx, dbeta_logits, dA_log, ddt_bias


def conv_forward(x, w):
    """x [B,T,C]; w [C,4] -> (silu(c), c)."""
    B, T, Ch = x.shape
    xp = F.pad(x, (0, 0, 3, 0))
    c = sum(xp[:, s:s + T] * w[:, s] for s in range(4))
    return F.silu(c), c


def conv_backward(x, w, c, dy):
    B, T, Ch = x.shape
    s = torch.sigmoid(c)
    dc = dy * s * (1 + c * (1 - s))
    dcp = F.pad(dc, (0, 0, 0, 3))
    dx = sum(dcp[:, 3 - s_:3 - s_ + T] * w[:, s_] for s_ in range(4))
    xp = F.pad(x, (0, 0, 3, 0))
    dw = torch.stack([(dc * xp[:, s_:s_ + T]).sum(dim=(0, 1)) for s_ in range(4)], -1)
    return dx, dw


def layer_forward_backward(inp: dict, *, conv: bool, lower_bound: float = -5.0,
                           scale: float | None = None, h0=None, dht=None):
    """Full staged forward + backward of one unpacked batch in the dtype of
    the inputs.  Returns outputs, gradients and every intermediate."""
    q_pre, k_pre, v_pre = inp["q"], inp["k"], inp["v"]
    B, T, H, D = q_pre.shape
    scale = D ** -0.5 if scale is None else scale
    HD = H * D
    if conv:
        posts, cs = [], []
        for x, w in ((q_pre, inp["conv_q"]), (k_pre, inp["conv_k"]), (v_pre, inp["conv_v"])):
            y, c = conv_forward(x.reshape(B, T, HD), w)
            posts.append(y.reshape(B, T, H, D))
            cs.append(c)
        q_in, k_in, v_in = posts
    else:
        q_in, k_in, v_in = q_pre, k_pre, v_pre
    qs, ks, vs, g, beta, qn, kn, z = prologue(q_in, k_in, v_in, inp["g"], inp["beta"],
                                              inp["A_log"], inp["dt_bias"], lower_bound, scale)
    ch = [_to_chunks(x, T) for x in (qs, ks, vs, g)]
    bch = _to_chunks(beta, T)
    it = intra(*ch, bch)
    S0 = torch.zeros(B, H, D, D, dtype=q_pre.dtype) if h0 is None else h0
    O, h, E, ST = state_forward(it, S0)
    o = _from_chunks(O, T)
    dO = _to_chunks(inp["do"], T)
    dST = torch.zeros_like(ST) if dht is None else dht
    dE, dh, dS0 = state_backward(it, dO, dST)
    dq, dk, dv, dg, dbeta = chunk_backward(*ch, bch, it, h, dh, E, dE, dO)
    dq, dk, dv, dg = (_from_chunks(x, T) for x in (dq, dk, dv, dg))
    dbeta = _from_chunks(dbeta, T)
    dq_in, dk_in, dg_logits, dbeta_logits, dA_log, ddt_bias = prologue_backward(
        q_in, k_in, qn, kn, z, beta, inp["A_log"], lower_bound, scale, dq, dk, dg, dbeta)
    grads = {"d_g": dg_logits, "d_beta": dbeta_logits, "d_A_log": dA_log,
             "d_dt_bias": ddt_bias, "d_h0": dS0}
    if conv:
        for name, x, w, c, dy in (("q", q_pre, inp["conv_q"], cs[0], dq_in),
                                  ("k", k_pre, inp["conv_k"], cs[1], dk_in),
                                  ("v", v_pre, inp["conv_v"], cs[2], dv)):
            dx, dw = conv_backward(x.reshape(B, T, HD), w, c, dy.reshape(B, T, HD))
            grads["d_" + name] = dx.reshape(B, T, H, D)
            grads["d_conv_" + name] = dw
    else:
        grads.update(d_q=dq_in, d_k=dk_in, d_v=dv)
    return dict(o=o, final_state=ST, grads=grads, intra=it, h=h, E=E, dE=dE, dh=dh)
