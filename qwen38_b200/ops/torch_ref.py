"""Plain-PyTorch definitions of every fused op (the numerical oracle).

Each function states the math of one kernel in ``qwen38_b200/csrc``; CUDA numerics tests
compare the kernel against these in fp32.  They also run the CPU (and gloo) paths of the
runtime.  Semantics follow the hybrid layer definitions the reference grafts onto TT-NN:

* ``(1+w)`` zero-centred RMSNorm for layer/q/k norms (``docker/qwen-c2-graft/graft/layer.py:110-111``)
* raw-weight gated RMSNorm times ``silu(z)`` for the GDN output (``graft/gdn/tp.py:1-7,694-710``)
* ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)`` (``graft/gdn/tp.py:610-614``)
* q/k L2 normalisation and ``Dk^-0.5`` query scale inside the delta rule
* partial RoPE on the first ``rope_dim`` channels, half-split rotation
* attention output times ``sigmoid(gate)`` (``graft/attention/tp.py:121-237``)
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, one_plus: bool = True) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    wf = w.float()
    y = y * ((1.0 + wf) if one_plus else wf)
    return y.to(x.dtype)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """residual += x; returns (norm(residual), residual). Residual kept in its own dtype."""
    r = (residual.float() + x.float()).to(residual.dtype)
    return rms_norm(r, w, eps), r


def gated_rms_norm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-head RMSNorm with raw weight, then times silu(z). o, z: [..., Dv]."""
    of = o.float()
    y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps)
    y = y * w.float()
    return (y * F.silu(z.float())).to(o.dtype)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + eps)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """Returns (g, beta) in fp32. a, b: [..., Nv]."""
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    beta = torch.sigmoid(b.float())
    return g, beta


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, window: torch.Tensor | None):
    """Depthwise causal conv (kernel K) followed by SiLU.

    x: [T, C] new inputs, w: [C, K], window: [K-1, C] previous inputs (zeros if None).
    Returns (y [T, C] fp32, new_window [K-1, C] in x's dtype)."""
    T, C = x.shape
    K = w.shape[1]
    if window is None:
        window = torch.zeros(K - 1, C, dtype=x.dtype, device=x.device)
    full = torch.cat([window.to(x.dtype), x], 0).float()            # [T+K-1, C]
    wf = w.float()
    y = torch.zeros(T, C, dtype=torch.float32, device=x.device)
    for j in range(K):
        y = y + full[j:j + T] * wf[:, j]
    return F.silu(y), full[T:].to(x.dtype) if K > 1 else full[:0].to(x.dtype)


def gdn_recurrent(q, k, v, g, beta, state):
    """Sequential gated delta rule.

    q, k: [T, H, Dk] (already L2-normalised, q already scaled); v: [T, H, Dv];
    g, beta: [T, H]; state: [H, Dk, Dv] fp32 (updated copy returned).
    Returns (o [T, H, Dv] fp32, state)."""
    S = state.float().clone()
    T = q.shape[0]
    outs = []
    for t in range(T):
        S = S * torch.exp(g[t].float())[:, None, None]
        kv = torch.einsum("hk,hkv->hv", k[t].float(), S)
        delta = (v[t].float() - kv) * beta[t].float()[:, None]
        S = S + torch.einsum("hk,hv->hkv", k[t].float(), delta)
        outs.append(torch.einsum("hk,hkv->hv", q[t].float(), S))
    return torch.stack(outs, 0), S


def gdn_chunked(q, k, v, g, beta, state, chunk: int = 64):
    """Chunked (WY-form) gated delta rule; same contract as ``gdn_recurrent``.

    Within a chunk of length C with cumulative log-decay G:
      A = strictly-lower( -(beta k) k^T * exp(G_i - G_j) ), T = (I - A)^-1 (forward substitution),
      U = T (beta v), W = T (beta k exp(G)), then per chunk
      V' = U - W S, O = (q exp(G)) S + tril(q k^T exp(G_i - G_j)) V',
      S <- exp(G_C) S + (k exp(G_C - G))^T V'.
    """
    T, H, Dk = k.shape
    Dv = v.shape[-1]
    S = state.float().clone()
    out = torch.zeros(T, H, Dv, dtype=torch.float32, device=q.device)
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        C = c1 - c0
        qc = q[c0:c1].float().transpose(0, 1)          # [H, C, Dk]
        kc = k[c0:c1].float().transpose(0, 1)
        vc = v[c0:c1].float().transpose(0, 1)          # [H, C, Dv]
        gc = g[c0:c1].float().transpose(0, 1)          # [H, C]
        bc = beta[c0:c1].float().transpose(0, 1)
        G = torch.cumsum(gc, -1)                        # [H, C]
        diff = G[:, :, None] - G[:, None, :]            # [H, C, C]
        lower = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device), -1)
        decay = torch.where(lower, torch.exp(torch.where(lower, diff, torch.zeros_like(diff))),
                            torch.zeros_like(diff))
        kb = kc * bc[..., None]
        A = -(kb @ kc.transpose(-1, -2)) * decay        # strictly lower
        Tm = torch.eye(C, device=q.device).expand(H, C, C).clone()
        for i in range(1, C):
            Tm[:, i, :i] = Tm[:, i, :i] + (A[:, i, :i, None] * Tm[:, :i, :i]).sum(1)
        U = Tm @ (vc * bc[..., None])
        W = Tm @ (kb * torch.exp(G)[..., None])
        Vp = U - W @ S
        incl = torch.tril(torch.ones(C, C, dtype=torch.bool, device=q.device))
        dq = torch.where(incl, torch.exp(torch.where(incl, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
        O = (qc * torch.exp(G)[..., None]) @ S + ((qc @ kc.transpose(-1, -2)) * dq) @ Vp
        out[c0:c1] = O.transpose(0, 1)
        GC = G[:, -1]
        S = torch.exp(GC)[:, None, None] * S + (kc * torch.exp(GC[:, None] - G)[..., None]).transpose(-1, -2) @ Vp
    return out, S


def rope_cos_sin(positions: torch.Tensor, rope_dim: int, theta: float, inv_freq: torch.Tensor | None = None,
                 scaling: float = 1.0):
    """cos/sin tables [T, rope_dim] (half-split layout: freqs repeated twice)."""
    if inv_freq is None:
        inv_freq = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float32) / rope_dim))
    ang = positions.float()[:, None] * inv_freq.to(positions.device)[None, :]
    emb = torch.cat([ang, ang], -1)
    return torch.cos(emb) * scaling, torch.sin(emb) * scaling


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; rotates the first cos.shape[-1] channels (half-split)."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd].float(), x[..., rd:]
    h = rd // 2
    rot = torch.cat([-xr[..., h:], xr[..., :h]], -1)
    y = xr * cos[:, None, :] + rot * sin[:, None, :]
    return torch.cat([y.to(x.dtype), xp], -1)


def attention(q, k, v, q_pos, k_pos, scale: float, causal: bool = True, window: int = 0):
    """GQA attention. q: [T, Hq, D], k/v: [S, Hkv, D]; q_pos [T], k_pos [S].
    A query at position p sees keys at positions <= p (causal) or all keys; with ``window`` > 0
    only keys k with p - k < window (the windowed drafter's mask, ``scripts/ci/draft_attention.py:14``)."""
    Hq, Hkv = q.shape[1], k.shape[1]
    rep = Hq // Hkv
    kf = k.float().repeat_interleave(rep, 1)
    vf = v.float().repeat_interleave(rep, 1)
    s = torch.einsum("thd,shd->hts", q.float(), kf) * scale
    if causal:
        mask = k_pos[None, :] > q_pos[:, None]
        s = s.masked_fill(mask[None], float("-inf"))
    if window > 0:
        mask = (q_pos[:, None] - k_pos[None, :]) >= window
        s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("hts,shd->thd", p, vf)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return (F.silu(gate.float()) * up.float()).to(gate.dtype)


def markov_select(base_logits: torch.Tensor, anchor: int, pred: torch.Tensor, succ: torch.Tensor):
    """Sequential Markov-biased greedy selection (``scripts/ci/dspark_markov.py:4-29``).

    base_logits [P, V]; pred/succ [V, R].  Step i scores ``base[i] + pred[prev] . succ^T`` and
    takes the argmax, which becomes ``prev`` for step i+1."""
    prev = int(anchor)
    out = []
    for i in range(base_logits.shape[0]):
        bias = succ.float() @ pred[prev].float()
        prev = int(torch.argmax(base_logits[i].float() + bias).item())
        out.append(prev)
    return out


def yarn_inv_freq(head_dim: int, theta: float, factor: float, beta_fast: float, beta_slow: float,
                  original_max: int):
    """YaRN inverse frequencies and attention scaling (the published YaRN method,
    as pinned for the drafter in ``scripts/ci/dspark_rope_tables.py:8-32``)."""
    def correction(rot):
        return head_dim * math.log(original_max / (rot * 2 * math.pi)) / (2 * math.log(theta))

    low = max(math.floor(correction(beta_fast)), 0)
    high = min(math.ceil(correction(beta_slow)), head_dim - 1)
    if high == low:
        high = low + 1e-3
    ramp = ((torch.arange(head_dim // 2, dtype=torch.float32) - low) / (high - low)).clamp(0, 1)
    extrap = 1 - ramp
    wl = theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    inv = (1 / (factor * wl)) * (1 - extrap) + (1 / wl) * extrap
    return inv, 1 + 0.1 * math.log(factor)


# ---------------------------------------------------------------------------- sampling noise
_M64 = (1 << 64) - 1


def _i64(c: int) -> int:
    """An unsigned 64-bit constant as the int64 with the same bits."""
    return c - (1 << 64) if c >= 1 << 63 else c


def _shr(z: torch.Tensor, k: int) -> torch.Tensor:
    """Logical right shift of int64 bit patterns."""
    return (z >> k) & ((1 << (64 - k)) - 1)


def mix64(z: torch.Tensor) -> torch.Tensor:
    """SplitMix64 finaliser (Steele, Lea, Flood, OOPSLA 2014) on int64 bit patterns (wrapping)."""
    z = (z ^ _shr(z, 30)) * _i64(0xBF58476D1CE4E5B9)
    z = (z ^ _shr(z, 27)) * _i64(0x94D049BB133111EB)
    return z ^ _shr(z, 31)


def gumbel_noise(key: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Gumbel(0, 1) noise [rows, n] from per-row keys [rows] and global indices [n]: the same
    counter-based construction as the device kernels (24-bit uniforms in (0, 1))."""
    h = mix64(key.long()[:, None] ^ mix64(index.long()[None, :] + _i64(0x9E3779B97F4A7C15)))
    u = (_shr(h, 40).double() + 0.5) / 16777216.0
    return (-torch.log(-torch.log(u))).float()


def sample_key(seed: int, position: int) -> int:
    """Noise key of one sampled token: a mix of the request seed and the token position, as int64."""
    z = torch.tensor([(seed * 0x9E3779B97F4A7C15 + position) & _M64], dtype=torch.uint64).view(torch.int64)
    return int(mix64(z)[0])


def draft_conv(x, dyn, tap0: int, base, group: int):
    """Dynamic grouped causal convolution of the windowed drafter (``scripts/ci/draft_convolution.py:17-37``):
    y[r, c] = (base[0, c] + dyn[r, tap0, c // group]) x[r, c] + (base[1, c] + dyn[r, tap0 + 1, c // group]) x[r - 1, c],
    x[-1] = 0, fp32 inputs rounded to bf16 first, the four products summed in that order in fp32."""
    R, H = x.shape
    G = H // group
    x0 = x.to(torch.bfloat16).float()
    x1 = torch.cat([torch.zeros_like(x0[:1]), x0[:-1]])
    d0 = dyn[:, tap0 * G:(tap0 + 1) * G].float().repeat_interleave(group, -1)
    d1 = dyn[:, (tap0 + 1) * G:(tap0 + 2) * G].float().repeat_interleave(group, -1)
    b = base.float().reshape(2, H)
    y = b[0] * x0
    y = y + d0 * x0
    y = y + b[1] * x1
    return y + d1 * x1


def greedy_select(feats, cand, unary, anchor: int, pred, succ):
    """fp64 greedy path through the candidates of rows 1..R-1 (``scripts/ci/draft_selector.py:37-56``):
    score(c) = unary[i, c] + sum_k pred[prev, k] f[i, k] succ[c, k], first maximum wins, prev starts at
    the anchor.  Returns (ids [R-1], per-row score vectors [R-1, C])."""
    prev = int(anchor)
    ids, rows = [], []
    for i in range(1, cand.shape[0]):
        c = cand[i].long().cpu()
        e = (pred[prev].double().cpu()[None, :] * feats[i].double().cpu()[None, :] * succ[c].double().cpu()).sum(-1)
        sc = unary[i].double().cpu() + e
        prev = int(c[int(torch.argmax(sc))])
        ids.append(prev)
        rows.append(sc)
    return torch.tensor(ids, dtype=torch.int64), torch.stack(rows)
