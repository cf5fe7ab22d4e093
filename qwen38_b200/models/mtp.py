"""Multi-token-prediction (MTP) head used as a drafter.

The checkpoint's own MTP module (``speculative-decoding/harness/mtp_module.py:46-110``): history
row p combines the target's last decoder-layer output h_p with the token that follows it,

    x   = fc(concat(rmsnorm_e(embed(token_{p+1})), rmsnorm_h(h_p)))     # [2H] -> [H]
    x  += attention(rmsnorm_in(x))        # one gated full-attention layer with its own KV history
    x  += mlp(rmsnorm_post(x))
    out = rmsnorm_final(x)  ->  shared LM head  ->  token_{p+2}

Multi-step proposals chain: the MTP output of row p is the hidden input of row p+1, with the
proposed token as its embedding input.  Norms are zero-centred (``1+w``) like the target's.

Same driver interface as the block drafter: ``taps`` (the target's last layer), ``append(feats,
pos, slot, next_tokens)`` publishes committed rows with their successor tokens, and
``propose(anchor, slot)`` returns the chained proposals.  Tensor parallel: the MTP
layer's attention and MLP are sharded like the target's, ``fc`` is replicated.
"""
from __future__ import annotations

import torch

from ..config import DrafterConfig, ModelConfig
from .target import GU_BLOCK, HybridTarget, pack_attn, pack_mlp


def mtp_shapes(cfg: ModelConfig) -> dict:
    h, d = cfg.hidden_size, cfg.head_dim
    p = "mtp.layers.0."
    out = {
        "mtp.fc.weight": (h, 2 * h),
        "mtp.pre_fc_norm_embedding.weight": (h,),
        "mtp.pre_fc_norm_hidden.weight": (h,),
        "mtp.norm.weight": (h,),
        p + "input_layernorm.weight": (h,),
        p + "post_attention_layernorm.weight": (h,),
        p + "self_attn.q_proj.weight": (2 * cfg.num_attention_heads * d, h),
        p + "self_attn.k_proj.weight": (cfg.num_key_value_heads * d, h),
        p + "self_attn.v_proj.weight": (cfg.num_key_value_heads * d, h),
        p + "self_attn.o_proj.weight": (h, cfg.num_attention_heads * d),
        p + "self_attn.q_norm.weight": (d,),
        p + "self_attn.k_norm.weight": (d,),
        p + "mlp.gate_proj.weight": (cfg.intermediate_size, h),
        p + "mlp.up_proj.weight": (cfg.intermediate_size, h),
        p + "mlp.down_proj.weight": (h, cfg.intermediate_size),
    }
    return out


def random_mtp_source(cfg: ModelConfig, seed: int = 2):
    from ..checkpoint import RandomSource
    return RandomSource(mtp_shapes(cfg), seed=seed)


class MTPDrafter:
    def __init__(self, src, target: HybridTarget, *, steps: int = 3, slots: int = 1, max_context: int | None = None):
        cfg = target.cfg
        self.cfg, self.target = cfg, target
        self.ops, self.comm = target.ops, target.comm
        self.device, self.dtype = target.device, target.dtype
        self.tp, r = target.tp, target.rank
        self.eps = cfg.rms_norm_eps
        self.P = steps
        # driver interface: one tap (the target's last decoder layer), blocks of steps+1 rows
        self.dcfg = DrafterConfig(hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                                  num_hidden_layers=1, num_attention_heads=cfg.num_attention_heads,
                                  num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                                  taps=[cfg.num_hidden_layers - 1], block_rows=steps + 1)
        dev, dt = self.device, self.dtype
        f32 = dict(device=dev, dtype=torch.float32)
        one = lambda n: (1.0 + src.get(n, **f32).float()).contiguous()
        self.fc = self.ops.prepare_weight(src.get("mtp.fc.weight", device=dev, dtype=dt).contiguous())
        self.norm_e = one("mtp.pre_fc_norm_embedding.weight")
        self.norm_h = one("mtp.pre_fc_norm_hidden.weight")
        self.norm_f = one("mtp.norm.weight")
        pfx = "mtp.layers.0."
        L = pack_attn(src, 0, cfg, self.tp, r, dev, dt, prefix=pfx)
        L.update(pack_mlp(src, 0, cfg, self.tp, r, dev, dt, prefix=pfx))
        for key in ("w_in", "w_out", "w_gu", "w_down"):
            L[key] = self.ops.prepare_weight(L[key])
        L["in_norm"] = one(pfx + "input_layernorm.weight")
        L["post_norm"] = one(pfx + "post_attention_layernorm.weight")
        self.L = L
        H, Hkv, D = L["dims"]
        self.max_context = max_context or target.rt.max_context
        cap = self.max_context + 2 * (steps + 2)
        self.slots = slots
        # [slot, layer (one), row, kv head, dim]: the block drafter's layout, so prefix checkpoints
        # snapshot and restore either drafter the same way
        self.kctx_all = torch.zeros(slots, 1, cap, Hkv, D, device=dev, dtype=dt)
        self.vctx_all = torch.zeros(slots, 1, cap, Hkv, D, device=dev, dtype=dt)
        self.positions = [0] * slots         # MTP history rows written so far
        self._last_hidden = [None] * slots   # target hidden of the newest committed row

    # ------------------------------------------------------------------ layer
    def _layer(self, tokens, hidden, positions, slot, write_only=False):
        """Rows (embed(tokens[i]), hidden[i]) at ``positions`` -> normed output rows [n, H]."""
        ops, L = self.ops, self.L
        e = ops.rms_norm(ops.embedding(tokens, self.target.embed), self.norm_e, self.eps, self.dtype)
        h = ops.rms_norm(hidden, self.norm_h, self.eps, self.dtype)
        x = ops.linear(torch.cat([e, h], -1).contiguous(), self.fc, out_dtype=torch.float32)
        a_in = ops.rms_norm(x, L["in_norm"], self.eps, self.dtype)
        proj = ops.linear(a_in, L["w_in"])
        q, gate = ops.attn_prep(proj, L["qn"], L["kn"], self.target.inv_freq, 1.0, self.cfg.rope_dim, L["dims"],
                                self.eps, positions, self.kctx_all[slot, 0], self.vctx_all[slot, 0], None, 0)
        if write_only:
            return None
        o = ops.attn_decode(q, gate, self.kctx_all[slot, 0], self.vctx_all[slot, 0], None, positions, 0, self.dtype)
        self._row_par_add(o, L["w_out"], x)
        f_in = self.target.norm(x, L["post_norm"], self.eps)
        gu = ops.linear_swiglu(f_in, L["w_gu"], GU_BLOCK)
        self._row_par_add(gu, L["w_down"], x)
        self.target.settle(x)             # x is read raw as the next step's hidden input
        return x

    def _row_par_add(self, h, w, x):
        self.target._row_parallel(h, w, x)      # same collectives as the target's out-projections

    # ------------------------------------------------------------------ driver interface
    # History row p holds (embed(token_{p+1}), h_p) at rotary / cache position p, so every committed
    # target row p has its MTP row; the newest one (whose successor token is the current seed)
    # starts each proposal chain.
    def reset(self, slot: int = 0):
        self.positions[slot] = 0
        self._last_hidden[slot] = None

    @torch.no_grad()
    def append(self, feats: torch.Tensor, pos: int, slot: int = 0, next_tokens=None):
        """Publish committed target rows pos..pos+n-1 (``feats``: their last-layer outputs) whose
        successor tokens are ``next_tokens``: writes MTP history rows pos..pos+n-1."""
        n = feats.shape[0]
        if next_tokens is None or len(next_tokens) < n:
            raise ValueError("the MTP drafter needs the committed successor of every published row")
        if pos != self.positions[slot]:
            raise ValueError(f"MTP history at {self.positions[slot]}, publication at {pos}")
        if pos + n + self.P + 1 > self.kctx_all.shape[2]:
            raise ValueError("MTP history capacity exceeded")
        hid = feats[:, -self.cfg.hidden_size:].float()
        toks = torch.as_tensor([int(t) for t in next_tokens[:n]], dtype=torch.long, device=self.device)
        positions = torch.arange(pos, pos + n, device=self.device, dtype=torch.int32)
        self._layer(toks, hid, positions, slot, write_only=True)
        self.positions[slot] = pos + n
        self._last_hidden[slot] = hid[n - 1:n].clone()

    @torch.no_grad()
    def propose(self, anchor: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """``steps`` chained proposals after ``anchor`` (the seed: successor of the newest row)."""
        r0 = self.positions[slot] - 1
        if r0 < 0:
            raise ValueError("propose before any publication")
        hidden = self._last_hidden[slot]
        tok = anchor.reshape(1).long()
        out = []
        for i in range(self.P):
            positions = torch.full((1,), r0 + i, device=self.device, dtype=torch.int32)
            x = self._layer(tok, hidden, positions, slot)
            hn = self.ops.rms_norm(x, self.norm_f, self.eps, self.dtype)
            val, idx = self.ops.lm_head_argmax(hn, self.target.lm_head, self.target.vocab_offset)
            if self.tp > 1:
                idx = self.comm.argmax_reduce(val, idx)
            tok = idx.reshape(1).long()
            out.append(tok)
            hidden = x                       # chain on the MTP's own output
        return torch.cat(out)

    def release_graphs(self):
        pass

    def close(self, slot: int = 0):
        self.reset(slot)
