"""Block drafter conditioned on target hidden states (DSpark family).

Forward, as pinned by the reference's CPU backbone (``scripts/ci/dspark_backbone_reference.py:46-110``)
and device drafter (``scripts/ci/dspark_device.py:34-103``):

1. Context rows: ``hidden_norm(fc(concat(tap features)))`` for every committed target position;
   each drafter layer projects them once into its K/V history (``k_norm`` + RoPE on K).
2. Block rows: target embeddings of ``[anchor, MASK, ..., MASK]`` (``P = block_rows - 1`` rows)
   at positions ``pos .. pos+P-1``; ``anchor`` is the committed seed at ``pos``.
3. Each layer: RMSNorm, q/k/v projections (q/k per-head RMSNorm, YaRN RoPE), attention of every
   block row over the whole history plus every block row (no causal mask inside the block),
   ``o_proj`` residual, SwiGLU residual.  Norm weights multiply directly (no ``1+w``).
4. Final norm, the target's (shared) LM head, then the sequential Markov selector: step i
   scores ``logits[i] + pred[prev] . succ^T`` and takes the argmax (``scripts/ci/dspark_markov.py``).

Publication (``scripts/ci/dflash_request_runtime.py:69-103``): after a commit, the accepted rows'
tap features are projected and appended to the history (incremental, never re-projected).

Tensor parallel like the target: heads split, KV heads replicated past their count, ``fc``
row-parallel over its input features, ``o_proj``/``down`` row-parallel, vocab-parallel head and
successor table with a cross-rank argmax per Markov step.
"""
from __future__ import annotations

import torch

from ..config import DrafterConfig
from ..ops import torch_ref as R
from .target import GU_BLOCK, HybridTarget


def _heads_split(n_heads, n_kv, tp, r):
    hl = n_heads // tp
    if tp > n_kv:
        return hl, 1, [r * n_kv // tp]
    kl = n_kv // tp
    return hl, kl, list(range(r * kl, (r + 1) * kl))


class BlockDrafter:
    def __init__(self, dcfg: DrafterConfig, src, target: HybridTarget, *, max_context: int | None = None,
                 slots: int = 1):
        self.dcfg, self.target = dcfg, target
        self.ops, self.comm = target.ops, target.comm
        self.device, self.dtype = target.device, target.dtype
        tp, r = target.tp, target.rank
        self.tp = tp
        H, Dh = dcfg.hidden_size, dcfg.head_dim
        if H != target.cfg.hidden_size:
            raise ValueError("drafter width must equal the target hidden size (shared embedding/head)")
        if dcfg.num_attention_heads % tp or dcfg.intermediate_size % (tp * GU_BLOCK):
            raise ValueError("drafter heads / intermediate do not divide by TP")
        self.eps = dcfg.rms_norm_eps
        self.P = dcfg.proposals
        self.mask_id = dcfg.mask_id(target.cfg.vocab_size)
        dev, dt = self.device, self.dtype
        f32 = lambda n: src.get(n, device=dev, dtype=torch.float32).float().contiguous()
        get = lambda n: src.get(n, device=dev, dtype=dt)
        nt = len(dcfg.taps)
        kin = nt * H
        if kin % tp:
            raise ValueError("fc input width must divide by TP")
        kl = kin // tp
        fc = get("fc.weight")
        self.fc = self.ops.prepare_weight(fc[:, r * kl:(r + 1) * kl].contiguous())
        del fc
        self.fc_k = (r * kl, kl)
        self.hidden_norm = f32("hidden_norm.weight")
        self.norm = f32("norm.weight")
        hl, kvl, kv_heads = _heads_split(dcfg.num_attention_heads, dcfg.num_key_value_heads, tp, r)
        self.heads = (hl, kvl, Dh)
        il = dcfg.intermediate_size // tp
        self.layers = []
        for l in range(dcfg.num_hidden_layers):
            p = f"layers.{l}."
            wq = get(p + "self_attn.q_proj.weight")[r * hl * Dh:(r + 1) * hl * Dh]
            wk = get(p + "self_attn.k_proj.weight").view(dcfg.num_key_value_heads, Dh, H)[kv_heads].reshape(-1, H)
            wv = get(p + "self_attn.v_proj.weight").view(dcfg.num_key_value_heads, Dh, H)[kv_heads].reshape(-1, H)
            g = get(p + "mlp.gate_proj.weight")[r * il:(r + 1) * il]
            u = get(p + "mlp.up_proj.weight")[r * il:(r + 1) * il]
            gu = torch.stack([g.reshape(il // GU_BLOCK, GU_BLOCK, H), u.reshape(il // GU_BLOCK, GU_BLOCK, H)], 1)
            pw = self.ops.prepare_weight
            self.layers.append(dict(
                w_qkv=pw(torch.cat([wq, wk, wv], 0).contiguous()),
                w_kv=pw(torch.cat([wk, wv], 0).contiguous()),
                w_o=pw(get(p + "self_attn.o_proj.weight")[:, r * hl * Dh:(r + 1) * hl * Dh].contiguous()),
                qn=f32(p + "self_attn.q_norm.weight"), kn=f32(p + "self_attn.k_norm.weight"),
                in_norm=f32(p + "input_layernorm.weight"), post_norm=f32(p + "post_attention_layernorm.weight"),
                w_gu=pw(gu.reshape(2 * il, H).contiguous()),
                w_down=pw(get(p + "mlp.down_proj.weight")[:, r * il:(r + 1) * il].contiguous()),
            ))
        vl = target.widths["vocab"]
        self.pred = get("markov_head.markov_w1.weight").contiguous()                 # [V, R] replicated
        self.succ = get("markov_head.markov_w2.weight")[r * vl:(r + 1) * vl].contiguous()  # [V_l, R]
        inv, scale = R.yarn_inv_freq(Dh, dcfg.rope_theta, dcfg.yarn_factor, dcfg.yarn_beta_fast,
                                     dcfg.yarn_beta_slow, dcfg.yarn_original_max_position)
        self.inv_freq, self.rope_scale = inv.to(dev), scale
        self.max_context = max_context or target.rt.max_context
        cap = self.max_context + 2 * dcfg.block_rows
        # one projected K/V history per slot (a request being served owns one slot)
        self.slots = slots
        self.kctx_all = torch.zeros(slots, dcfg.num_hidden_layers, cap, kvl, Dh, device=dev, dtype=dt)
        self.vctx_all = torch.zeros(slots, dcfg.num_hidden_layers, cap, kvl, Dh, device=dev, dtype=dt)
        self.positions = [0] * slots
        self.use_graphs = target.use_graphs
        self._graphs = {}
        self._init_propose_buffers(self.P)

    def _init_propose_buffers(self, rows: int):
        """Static anchor / position buffers of the captured propose step (``rows`` block rows)."""
        dev, slots = self.device, self.slots
        self.rows = rows
        self._anchor_buf = torch.zeros(slots, 1, dtype=torch.long, device=dev)
        self._pos_buf = torch.zeros(slots, rows, dtype=torch.int32, device=dev)
        self._pos_host = torch.zeros(rows, dtype=torch.int32).pin_memory() if dev.type == "cuda" else None

    # slot-0 views (single-stream API)
    @property
    def kctx(self):
        return self.kctx_all[0]

    @property
    def vctx(self):
        return self.vctx_all[0]

    @property
    def position(self):
        return self.positions[0]

    @position.setter
    def position(self, v):
        self.positions[0] = v

    # -------------------------------------------------------------------------------- helpers
    def _row_par(self, h, w):
        part = self.ops.linear(h, w, out_dtype=torch.float32)
        if self.tp > 1:
            self.comm.all_reduce_(part)
        return part

    def _row_par_add(self, h, w, x):
        """x += h @ w^T summed over ranks."""
        if self.tp == 1:
            self.target.local_row_parallel(h, w, x)     # completed by the next norm of x
        elif self.target.fused_ar and self.comm.fused_fits(*x.shape):
            self.target.push_row_parallel(h, w, x)      # completed by the next norm of x
        elif hasattr(self.comm, "slot_out") and self.comm.fits(*x.shape):
            slot, part = self.comm.slot_out(*x.shape)
            self.ops.linear(h, w, out=part)
            self.comm.reduce_slot_add(slot, x)
        else:
            x += self._row_par(h, w)
        return x

    def _context_rows(self, feats):
        """fc (row-parallel over tap features) then hidden_norm -> [S, H] in activation dtype."""
        k0, kl = self.fc_k
        part = self._row_par(feats[:, k0:k0 + kl].contiguous() if self.tp > 1 else feats, self.fc)
        return self.ops.rms_norm(part, self.hidden_norm, self.eps, self.dtype)

    # -------------------------------------------------------------------------------- history
    def reset(self, slot: int = 0):
        self.positions[slot] = 0

    @torch.no_grad()
    def append(self, feats: torch.Tensor, pos: int, slot: int = 0, next_tokens=None):
        """Project ``feats`` [n, taps*H] (target rows at positions pos..pos+n-1) into every layer's
        K/V history of ``slot``."""
        if pos != self.positions[slot]:
            raise ValueError(f"drafter history at {self.positions[slot]}, publication at {pos}")
        n = feats.shape[0]
        if pos + n > self.max_context:
            raise ValueError("drafter history capacity exceeded")
        positions = torch.arange(pos, pos + n, device=self.device, dtype=torch.int32)
        self.append_device(feats, positions, slot)
        self.positions[slot] = pos + n

    def append_device(self, feats: torch.Tensor, positions: torch.Tensor, slot: int):
        """The device half of ``append`` (capturable: positions come from a device tensor)."""
        ctx = self._context_rows(feats)
        hl, kvl, Dh = self.heads
        for l, L in enumerate(self.layers):
            kv = self.ops.linear(ctx, L["w_kv"])
            self.ops.kv_append(kv, L["kn"], self.inv_freq, self.rope_scale, Dh, kvl, Dh, self.eps, positions,
                               self.kctx_all[slot, l], self.vctx_all[slot, l])

    # -------------------------------------------------------------------------------- propose
    @torch.no_grad()
    def forward_block(self, anchor: torch.Tensor, positions: torch.Tensor | None = None, slot: int = 0):
        """Block forward at the current history frontier; returns local-vocab logits [P, V_l]."""
        P, pos = self.P, self.positions[slot]
        hl, kvl, Dh = self.heads
        ids = torch.full((P,), self.mask_id, dtype=torch.long, device=self.device)
        ids[:1] = anchor.reshape(1)
        h = self.ops.embedding(ids, self.target.embed).float()
        if positions is None:
            positions = torch.arange(pos, pos + P, device=self.device, dtype=torch.int32)
        norm = self.target.norm
        for l, L in enumerate(self.layers):
            hn = norm(h, L["in_norm"], self.eps)
            qkv = self.ops.linear(hn, L["w_qkv"])
            o = self.ops.draft_block_attention(qkv, L["qn"], L["kn"], self.inv_freq, self.rope_scale, self.heads,
                                               self.eps, positions, self.kctx_all[slot, l],
                                               self.vctx_all[slot, l], self.dtype)
            self._row_par_add(o, L["w_o"], h)
            hn = norm(h, L["post_norm"], self.eps)
            gu = self.ops.linear_swiglu(hn, L["w_gu"], GU_BLOCK)
            self._row_par_add(gu, L["w_down"], h)
        hn = norm(h, self.norm, self.eps)
        return self.ops.linear(hn, self.target.lm_head, out_dtype=torch.float32)

    def _propose_eager(self, anchor, positions=None, slot: int = 0):
        logits = self.forward_block(anchor, positions, slot)
        return self.ops.markov_select(logits, anchor, self.pred, self.succ, self.target.vocab_offset,
                                      self.comm if self.tp > 1 else None)

    @torch.no_grad()
    def propose(self, anchor: torch.Tensor, slot: int = 0) -> torch.Tensor:
        """Returns P proposal ids (device int64) for the block after ``anchor`` (CUDA-graph replay
        with static anchor/position buffers when graphs are enabled)."""
        if not self.use_graphs:
            return self._propose_eager(anchor, None, slot)
        pos = self.positions[slot]
        if pos + self.rows > self.kctx_all.shape[2]:
            raise ValueError("drafter history capacity exceeded")
        ab, pb = self._anchor_buf[slot], self._pos_buf[slot]
        ab.copy_(anchor.reshape(1))
        self._pos_host.copy_(torch.arange(pos, pos + self.rows, dtype=torch.int32))
        pb.copy_(self._pos_host, non_blocking=True)
        if slot not in self._graphs:
            self._propose_eager(ab, pb, slot)          # warm-up
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            l0 = getattr(self.ops, "launches", 0)
            if hasattr(self.comm, "begin_capture"):
                self.comm.begin_capture()
            with torch.cuda.graph(g):
                out = self._propose_eager(ab, pb, slot)
            self._graphs[slot] = (g, out, getattr(self.ops, "launches", 0) - l0)
        g, out, n = self._graphs[slot]
        g.replay()
        if hasattr(self.ops, "launches"):
            self.ops.launches += n
        return out

    def release_graphs(self):
        self._graphs.clear()

    def close(self, slot: int = 0):
        self.positions[slot] = 0
