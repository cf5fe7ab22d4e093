"""fp32 PyTorch reference of the hybrid decoder (the oracle for the runtime and the kernels).

Layer math: pre-norm residual blocks ``x + mixer(norm(x))`` then ``h + mlp(norm(h))`` with a
GDN or gated-attention mixer chosen per ``layer_types`` (reference:
``docker/qwen-c2-graft/graft/layer.py:93-364``); the top-level model embeds, runs the stack,
applies the final norm and the LM head (``scripts/ci/fixtures/qwen36_model.py:24-137,495``).

It keeps a contiguous KV cache and exact sequential GDN state, so ``step`` over any split of a
sequence yields the same logits as one pass.  It consumes the HF-layout state dict written by
``qwen38_b200.checkpoint``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..config import LINEAR, ModelConfig
from ..ops import torch_ref as R


@dataclass
class RefState:
    pos: int = 0
    kv: dict = field(default_factory=dict)       # layer -> (K [S,Hkv,D], V [S,Hkv,D])
    rec: dict = field(default_factory=dict)      # layer -> [Nv, Dk, Dv] fp32
    conv: dict = field(default_factory=dict)     # layer -> [K-1, C]

    def clone(self) -> "RefState":
        return RefState(self.pos,
                        {k: (a.clone(), b.clone()) for k, (a, b) in self.kv.items()},
                        {k: v.clone() for k, v in self.rec.items()},
                        {k: v.clone() for k, v in self.conv.items()})


class ReferenceModel:
    def __init__(self, cfg: ModelConfig, sd: dict, dtype=torch.float32, chunked_gdn: bool = False,
                 gdn_chunk: int = 64):
        self.cfg = cfg
        self.dtype = dtype
        self.sd = {k: v.to(dtype) if v.is_floating_point() else v for k, v in sd.items()}
        self.chunked_gdn = chunked_gdn
        self.gdn_chunk = gdn_chunk

    def w(self, name):
        return self.sd[name]

    def new_state(self) -> RefState:
        return RefState()

    # ---------------------------------------------------------------- mixers
    def _gdn(self, i, x, st: RefState):
        c = self.cfg
        p = f"model.layers.{i}.linear_attn."
        T = x.shape[0]
        qkv = x @ self.w(p + "in_proj_qkv.weight").T
        z = x @ self.w(p + "in_proj_z.weight").T
        b = x @ self.w(p + "in_proj_b.weight").T
        a = x @ self.w(p + "in_proj_a.weight").T
        convw = self.w(p + "conv1d.weight").reshape(c.gdn_conv_dim, -1)
        y, st.conv[i] = R.causal_conv1d(qkv, convw, st.conv.get(i))
        kd, Nk, Nv, Dk, Dv = c.gdn_key_dim, c.linear_num_key_heads, c.linear_num_value_heads, \
            c.linear_key_head_dim, c.linear_value_head_dim
        q = y[:, :kd].reshape(T, Nk, Dk)
        k = y[:, kd:2 * kd].reshape(T, Nk, Dk)
        v = y[:, 2 * kd:].reshape(T, Nv, Dv)
        rep = Nv // Nk
        q = R.l2norm(q).repeat_interleave(rep, 1) * (Dk ** -0.5)
        k = R.l2norm(k).repeat_interleave(rep, 1)
        g, beta = R.gdn_gates(a, b, self.w(p + "A_log"), self.w(p + "dt_bias"))
        S = st.rec.get(i)
        if S is None:
            S = torch.zeros(Nv, Dk, Dv, dtype=torch.float32, device=x.device)
        if self.chunked_gdn and T > 1:
            o, S = R.gdn_chunked(q, k, v, g, beta, S, self.gdn_chunk)
        else:
            o, S = R.gdn_recurrent(q, k, v, g, beta, S)
        st.rec[i] = S
        o = R.gated_rms_norm(o.to(x.dtype), z.reshape(T, Nv, Dv), self.w(p + "norm.weight"), c.rms_norm_eps)
        return o.reshape(T, -1) @ self.w(p + "out_proj.weight").T

    def _attn(self, i, x, st: RefState, positions):
        c = self.cfg
        p = f"model.layers.{i}.self_attn."
        T = x.shape[0]
        H, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qg = (x @ self.w(p + "q_proj.weight").T).reshape(T, H, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(T, H * D)
        k = (x @ self.w(p + "k_proj.weight").T).reshape(T, Hkv, D)
        v = (x @ self.w(p + "v_proj.weight").T).reshape(T, Hkv, D)
        q = R.rms_norm(q, self.w(p + "q_norm.weight"), c.rms_norm_eps)
        k = R.rms_norm(k, self.w(p + "k_norm.weight"), c.rms_norm_eps)
        cos, sin = R.rope_cos_sin(positions, c.rope_dim, c.rope_theta)
        q = R.apply_rope(q, cos, sin)
        k = R.apply_rope(k, cos, sin)
        if i in st.kv:
            K, V = st.kv[i]
            K, V = torch.cat([K, k], 0), torch.cat([V, v], 0)
        else:
            K, V = k, v
        st.kv[i] = (K, V)
        kpos = torch.arange(K.shape[0], device=x.device)
        o = R.attention(q, K, V, positions, kpos, D ** -0.5, causal=True).to(x.dtype)
        o = o.reshape(T, H * D) * torch.sigmoid(gate.float()).to(x.dtype)
        return o @ self.w(p + "o_proj.weight").T

    def _mlp(self, i, x):
        p = f"model.layers.{i}.mlp."
        g = x @ self.w(p + "gate_proj.weight").T
        u = x @ self.w(p + "up_proj.weight").T
        return R.swiglu(g, u) @ self.w(p + "down_proj.weight").T

    # ---------------------------------------------------------------- forward
    @torch.no_grad()
    def step(self, tokens: torch.Tensor, st: RefState, taps=()):
        """Process ``tokens`` [T] at positions ``st.pos ..``; returns (logits [T, V] fp32,
        {tap: hidden [T, H]}, final normed hidden [T, H]).  Advances ``st``."""
        c = self.cfg
        T = tokens.shape[0]
        positions = torch.arange(st.pos, st.pos + T, device=tokens.device)
        x = self.w("model.embed_tokens.weight")[tokens]
        tapped = {}
        for i, lt in enumerate(c.layer_types):
            p = f"model.layers.{i}."
            h = R.rms_norm(x, self.w(p + "input_layernorm.weight"), c.rms_norm_eps)
            mix = self._gdn(i, h, st) if lt == LINEAR else self._attn(i, h, st, positions)
            x = x + mix
            h = R.rms_norm(x, self.w(p + "post_attention_layernorm.weight"), c.rms_norm_eps)
            x = x + self._mlp(i, h)
            if i in taps:
                tapped[i] = x.clone()
        st.pos += T
        hn = R.rms_norm(x, self.w("model.norm.weight"), c.rms_norm_eps)
        head = self.w("model.embed_tokens.weight") if c.tie_word_embeddings else self.w("lm_head.weight")
        return (hn @ head.T).float(), tapped, hn

    @torch.no_grad()
    def greedy(self, prompt: torch.Tensor, max_new_tokens: int, eos=None):
        st = self.new_state()
        logits, _, _ = self.step(prompt, st)
        out = [int(torch.argmax(logits[-1]))]
        while len(out) < max_new_tokens and (eos is None or out[-1] != eos):
            logits, _, _ = self.step(torch.tensor([out[-1]], device=prompt.device), st)
            out.append(int(torch.argmax(logits[-1])))
        return out
