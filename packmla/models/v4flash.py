"""DeepSeek-V4-Flash-shape model: MLA over one 512-wide latent with C4/C128 compressed sparse
attention, SWA, attention sinks, grouped output projection and sigmoid-routed MoE.

Reference behaviour: `srt/models/deepseek_v4.py`, `srt/layers/attention/dsv4/{compressor_v2,indexer}.py`
and `deepseek_v4_backend.py` of the reference's SGLang fork (third_party/README.md:275-279; the
fork sources are absent, so the layer internals below are packmla's own design constrained by
the shapes and contracts the reference records, see packmla/config.py).

Per layer (decode, B tokens of B different requests):
  h = rmsnorm(x);  [q_lora | kv] = h Wqkv_a;  q = rmsnorm(q_lora) Wq_b (heads x 512), tail RoPE
  kv -> Native record in the layer's SWA ring (norm kv_norm, RoPE at the token position)
  compressor (ratio 4 / 128): online-softmax pooling of h Wc_kv with gates h Wc_gate + ape;
     a completed group -> C4 record (Native or Packed store) / C128 record (Native)
  indexer: score(r) = sum_h w_h relu(q_idx_h . k_r), top-512 records (k_r FP8, pooled like kv)
  o = sparse MLA attention over [SWA ring ; selected C4 | all C128 records] with sink
  x += (o grouped-projected by Wo_a, then Wo_b)              -> TP all-reduce
  x += shared(rmsnorm(x)) + sum_k w_k expert_k(rmsnorm(x))   -> TP/EP all-reduce
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..config import EngineConfig, ModelConfig
from ..formats import abi, codec
from ..kv.pool import KVPool
from ..ops import attention as attn_ops
from ..ops import kv as kv_ops
from ..ops import indexer as idx_ops
from ..ops import moe as moe_ops
from ..ops import dense as dense_ops
from ..ops import fused as fused_ops


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return fused_ops.add_rmsnorm(x, w, eps)[1]


@dataclass
class StepMeta:
    """Per-step attention metadata shared by all layers of a kind (device tensors)."""

    positions: torch.Tensor  # [B] int64
    req_slots: torch.Tensor  # [B] int64
    swa_slots: torch.Tensor  # [B, 128] int32
    swa_len: torch.Tensor  # [B] int32
    swa_write: torch.Tensor  # [B] int64 ring slot of this token
    c4_phys: torch.Tensor  # [B, R4] int32 physical record of logical record r (or -1)
    c4_count: torch.Tensor  # [B] int64 complete C4 records visible to the query
    c4_write: torch.Tensor  # [B] int64 physical slot of the record completed now, else -1
    c128_slots: torch.Tensor  # [B, R128] int32 (masked by count)
    c128_pos: torch.Tensor  # [B, R128] int32
    c128_len: torch.Tensor  # [B] int32
    c128_write: torch.Tensor  # [B] int64
    no_rows: torch.Tensor  # [B, 0] int32 (layers without compressed records: an empty C4 list)
    zero_len: torch.Tensor  # [B] int32 zeros
    topk_len: torch.Tensor  # [B] int32 = index top-k
    positions_i32: torch.Tensor  # [B] int32


class V4FlashModel:
    def __init__(self, cfg: ModelConfig, weights: dict, pool: KVPool, comm=None):
        self.cfg = cfg
        # the model's own layer dicts: fusing and quantizing replace entries without touching the caller's
        self.W = {**weights, "layers": [dict(lw) for lw in weights["layers"]]}
        self.pool = pool
        self.comm = comm
        self.device = pool.device
        self.kv_format = pool.kv_format
        meta = weights["meta"]
        self.world = meta["world"]
        self.expert_base = meta["expert_base"]
        self.local_experts = meta["local_experts"]
        # DP attention: this rank serves its own requests with every head; only the routed experts are
        # split, and each MoE block exchanges tokens with the other ranks (all-gather in, reduce-scatter
        # out).  `dp_counts` (tokens of every rank in the current forward, set by the caller) sizes it.
        self.dp = bool(meta.get("dp_attention", False)) and self.world > 1
        self.dp_counts: list[int] | None = None
        attn_world = meta.get("attn_world", self.world)
        self.heads = cfg.num_heads // attn_world
        self.groups = cfg.o_groups // attn_world
        self.scale = 1.0 / math.sqrt(cfg.latent_dim)
        self.freqs = kv_ops.freq_table_f32(codec.rope_table(cfg.max_position, cfg.rope_theta)).to(self.device)
        self.r4max = pool.max_context // abi.C4_RATIO
        self.r128max = max(1, pool.max_context // abi.C128_RATIO)
        self.topk = min(cfg.index_topk, self.r4max)
        # fused output projection + all-reduce over peer memory (parallel.fused.FusedComm) when available
        self.ar_hook = getattr(comm, "gemm_all_reduce", None) if self.world > 1 and not self.dp else None
        self.moe_precision = "default"  # MXFP8 expert activations ("bf16": BF16 activations)
        # optional capture observer (packmla.training.data.capture): sees every C4 store and every decode
        # query of a C4 layer; None on the serving path
        self.observer = None
        self.adapter_ws = None
        if self.kv_format == "direct" and pool.ecfg.decode_impl == "adapter":
            rows = pool.max_requests * self.topk
            self.adapter_ws = torch.zeros(-(-rows // abi.RECORDS_PER_PAGE) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8,
                                          device=self.device)
        self.fused = [self._fuse_layer(i) for i in range(cfg.num_layers)]
        # MXFP8 dense projections (cfg.dense_format "fp8", csrc/dense_mx.cu); the router gate and the LM
        # head stay BF16, as in DeepSeek's FP8 checkpoints
        self.mx = None
        self.dense_ws = None
        if cfg.dense_format == "fp8":
            self.mx = [self._quantize_dense(i) for i in range(cfg.num_layers)]
            if self.device.type == "cuda":
                self.dense_ws = self._dense_workspace()
            self.ar_hook = None  # the fused GEMM + all-reduce takes BF16 weights

    def _fuse_layer(self, layer: int) -> dict:
        """Concatenate every projection of the normed residual into one weight per block.

        Attention block: [wqkv_a | wc_kv | wc_gate | wi_k | wi_kgate | wi_w] (the compressor and
        indexer parts only where the layer compresses); FFN block: [shared_w13 | gate].  The layer's
        named weights become row views of the concatenation, so no weight is stored twice.
        """
        cfg = self.cfg
        lw = self.W["layers"][layer]
        ratio = cfg.compress_ratios[layer]
        names = ["wqkv_a"]
        if ratio:
            names += ["wc_kv", "wc_gate"]
        if ratio == abi.C4_RATIO:
            names += ["wi_k", "wi_kgate", "wi_w"]
        out = {}
        for key, group in (("w_h", names), ("w_ffn", ["shared_w13", "gate"])):
            w = torch.cat([lw[n] for n in group]).contiguous()
            off = 0
            for n in group:
                rows = lw[n].shape[0]
                lw[n] = w[off:off + rows]
                out[n] = off
                off += rows
            out[key] = w
        return out

    def _quantize_dense(self, layer: int) -> dict:
        """MXFP8 weights of one layer's dense projections; their BF16 copies are dropped from the model.

        w_h: the fused attention input projection; wqi: [wq_b ; wi_q] (the q up-projection and, in C4
        layers, the indexer query share their input); wo_a: one [o_lora, heads_per_group x 512] matrix per
        output group; wo_b; shared_w13; shared_w2."""
        cfg = self.cfg
        lw = self.W["layers"][layer]
        fz = self.fused[layer]
        ratio = cfg.compress_ratios[layer]
        wq = torch.cat([lw["wq_b"], lw["wi_q"]]) if ratio == abi.C4_RATIO else lw["wq_b"]
        mx = {"w_h": dense_ops.quantize_weight(fz["w_h"]), "wqi": dense_ops.quantize_weight(wq),
              "wo_a": dense_ops.quantize_weight(lw["wo_a"].transpose(1, 2)),
              "wo_b": dense_ops.quantize_weight(lw["wo_b"]),
              "shared_w13": dense_ops.quantize_weight(lw["shared_w13"]),
              "shared_w2": dense_ops.quantize_weight(lw["shared_w2"])}
        gate = lw["gate"].clone()  # a view of the fused FFN weight: keep only the gate rows
        for n in ("wqkv_a", "wc_kv", "wc_gate", "wi_k", "wi_kgate", "wi_w", "wq_b", "wi_q", "wo_a", "wo_b",
                  "shared_w13", "shared_w2"):
            lw.pop(n, None)
        lw["gate"] = gate
        fz["w_h"] = fz["w_ffn"] = None
        return mx

    def _dense_workspace(self) -> "dense_ops.DenseWorkspace":
        """One workspace for every dense call of a decode step (at most the pool's request count) and of a
        prefill chunk."""
        cfg, ecfg = self.cfg, self.pool.ecfg
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        calls = []
        for T in {max(1, self.pool.max_requests + 1), max(1, ecfg.chunked_prefill_size)}:
            for mx in self.mx:
                for w in mx.values():
                    calls.append((T, w.n, w.k, w.batch))
        return dense_ops.DenseWorkspace.for_calls(calls, self.device, sms)

    def _dense(self, layer: int, name: str, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        w = self.mx[layer][name]
        ws = self.dense_ws
        if ws is not None and not ws.fits(x.shape[-2], w.k, w.n, w.batch):
            # larger than the engine's decode batch and prefill chunk (a direct model call): the growable
            # per-device workspace (never reached inside a captured decode step)
            ws = None
        return dense_ops.mx_linear(x, w, out=out, workspace=ws)

    def _proj_h(self, layer: int, h: torch.Tensor) -> torch.Tensor:
        """The fused attention input projection (q LoRA | latent | compressor | indexer parts)."""
        if self.mx is not None:
            return self._dense(layer, "w_h", h)
        return h @ self.fused[layer]["w_h"].T

    def _proj_q(self, layer: int, q_lora: torch.Tensor):
        """(q up-projection [T, heads x 512], indexer queries [T, index_heads x index_dim] or None)."""
        if self.mx is None:
            return q_lora @ self.W["layers"][layer]["wq_b"].T, None
        qq = self._dense(layer, "wqi", q_lora)
        hl = self.heads * self.cfg.latent_dim
        return qq[:, :hl], (qq[:, hl:] if self.cfg.compress_ratios[layer] == abi.C4_RATIO else None)

    # ------------------------------------------------------------------ helpers
    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.comm is None or self.world == 1 or self.dp:  # DP attention: the rank has every head
            return t
        return self.comm.all_reduce(t)

    def csa_planes(self, layer: int):
        p = self.pool
        if p.fp4_format is not None:
            return p.c4_fp4[layer], None
        if self.kv_format == "direct":
            return None, attn_ops.PackedPlanes(p.c4_values[layer], p.c4_bitmap[layer], p.c4_scales[layer])
        return p.c4_native[layer], None

    # ------------------------------------------------------------------ metadata
    def step_meta(self, positions: torch.Tensor, req_slots: torch.Tensor) -> StepMeta:
        """Decode metadata (graph-capturable: no host synchronization)."""
        dev = self.device
        p = self.pool
        B = positions.shape[0]
        W = self.cfg.window
        pos = positions.long()
        req = req_slots.long()
        ar = torch.arange(W, device=dev, dtype=torch.int64)
        swa_slots = (req[:, None] * W + ar[None]).int()
        swa_len = torch.clamp(pos + 1, max=W).int()
        swa_write = req * W + pos % W
        r = torch.arange(self.r4max, device=dev, dtype=torch.int64)
        pt = p.page_table[req]  # [B, pages]
        page = pt.gather(1, (r // abi.RECORDS_PER_PAGE).clamp(max=pt.shape[1] - 1)[None].expand(B, -1)).long()
        c4_phys = torch.where(page >= 0, page * abi.RECORDS_PER_PAGE + r % abi.RECORDS_PER_PAGE, -1)
        c4_count = (pos + 1) // abi.C4_RATIO
        rec = pos // abi.C4_RATIO
        done4 = (pos % abi.C4_RATIO) == abi.C4_RATIO - 1
        w4 = c4_phys.gather(1, rec.clamp(max=self.r4max - 1)[:, None])[:, 0]
        c4_write = torch.where(done4 & (rec < self.r4max), w4, torch.full_like(w4, -1))
        r2 = torch.arange(self.r128max, device=dev, dtype=torch.int64)
        ct = p.c128_table[req]
        page2 = ct.gather(1, (r2 // abi.RECORDS_PER_PAGE).clamp(max=ct.shape[1] - 1)[None].expand(B, -1)).long()
        phys2 = torch.where(page2 >= 0, page2 * abi.RECORDS_PER_PAGE + r2 % abi.RECORDS_PER_PAGE, -1)
        n128 = (pos + 1) // abi.C128_RATIO
        c128_slots = torch.where(r2[None] < n128[:, None], phys2, torch.full_like(phys2, -1)).int()
        c128_pos = (r2 * abi.C128_RATIO).int()[None].expand(B, -1).contiguous()
        rec2 = pos // abi.C128_RATIO
        done2 = (pos % abi.C128_RATIO) == abi.C128_RATIO - 1
        w2 = phys2.gather(1, rec2.clamp(max=self.r128max - 1)[:, None])[:, 0]
        c128_write = torch.where(done2 & (rec2 < self.r128max), w2, torch.full_like(w2, -1))
        c128_len = torch.full((B,), self.r128max, dtype=torch.int32, device=dev)
        return StepMeta(pos, req, swa_slots, swa_len, swa_write, c4_phys.int(), c4_count, c4_write,
                        c128_slots, c128_pos, c128_len, c128_write,
                        torch.empty((B, 0), dtype=torch.int32, device=dev),
                        torch.zeros(B, dtype=torch.int32, device=dev),
                        torch.full((B,), self.topk, dtype=torch.int32, device=dev), pos.int())

    # ------------------------------------------------------------------ compressor
    def _compress_decode(self, layer: int, y: torch.Tensor, meta: StepMeta) -> None:
        """Pool this token into the layer's compressor (and indexer-key) state; store completed records.

        `y` is the attention block's fused projection; the compressor's (value | gate) columns and the
        indexer's (key | gate) columns are adjacent in it.
        """
        lw = self.W["layers"][layer]
        fz = self.fused[layer]
        ratio = self.cfg.compress_ratios[layer]
        pos = meta.positions
        L = self.cfg.latent_dim
        raw = fused_ops.comp_pool(y, fz["wc_kv"], L, lw["c_ape"], self.pool.comp_state[layer], meta.req_slots, pos)
        if ratio == abi.C4_RATIO:
            self._store_c4(layer, raw, meta.c4_write, (pos // ratio) * ratio)
            kraw = fused_ops.comp_pool(y, fz["wi_k"], self.cfg.index_dim, lw["i_ape"], self.pool.index_state[layer],
                                       meta.req_slots, pos)
            self._store_index_keys(layer, kraw, meta.c4_write)
        else:
            kv_ops.native_store(raw, lw["c_norm"], self.cfg.rms_eps, meta.c128_write, (pos // ratio) * ratio,
                                self.freqs, self.pool.c128_native[layer])

    def _store_c4(self, layer: int, raw: torch.Tensor, slots: torch.Tensor, rope_pos: torch.Tensor) -> None:
        lw = self.W["layers"][layer]
        p = self.pool
        if self.observer is not None:
            self.observer.observe_raw(layer, raw, slots)
        if p.fp4_format is not None:
            kv_ops.fp4_store(raw, lw["c_norm"], self.cfg.rms_eps, slots, rope_pos, self.freqs, p.c4_fp4[layer],
                             p.fp4_format == "direct")
        elif self.kv_format == "direct":
            kv_ops.packed_store(raw, lw["c_norm"], self.cfg.rms_eps, slots, p.c4_values[layer], p.c4_bitmap[layer],
                                p.c4_scales[layer])
        else:
            kv_ops.native_store(raw, lw["c_norm"], self.cfg.rms_eps, slots, rope_pos, self.freqs, p.c4_native[layer])

    def _store_index_keys(self, layer: int, kraw: torch.Tensor, slots: torch.Tensor) -> None:
        """FP8 index key + fp32 scale per completed record (rows with slot -1 are skipped)."""
        idx_ops.index_key_store(kraw, slots, self.pool.index_keys[layer], self.pool.index_scales[layer])

    # ------------------------------------------------------------------ indexer
    def _index_topk(self, layer: int, q_lora: torch.Tensor, y: torch.Tensor, phys: torch.Tensor,
                    count: torch.Tensor, r_limit: int, qi: torch.Tensor | None = None):
        """Top-k C4 records per query: returns (slots int32 [B,K], rope positions int32 [B,K]).  `qi`: the
        indexer queries [B, index_heads x index_dim] when the caller projected them already."""
        lw = self.W["layers"][layer]
        cfg = self.cfg
        B = q_lora.shape[0]
        qi = (q_lora @ lw["wi_q"].T) if qi is None else qi
        qi = qi.view(B, cfg.index_heads, cfg.index_dim)
        c = self.fused[layer]["wi_w"]
        wi = y[:, c:c + cfg.index_heads].float() * ((cfg.index_heads ** -0.5) * (cfg.index_dim ** -0.5))
        return idx_ops.index_select(qi.contiguous(), wi, self.pool.index_keys[layer], self.pool.index_scales[layer],
                                    phys, count, r_limit, min(self.topk, r_limit))

    # ------------------------------------------------------------------ layer
    def _attention_block(self, layer: int, h: torch.Tensor, meta: StepMeta) -> torch.Tensor:
        """Attention of the normed residual h [B, H] -> bf16 [B, H] (all-reduced over TP)."""
        cfg = self.cfg
        lw = self.W["layers"][layer]
        B = h.shape[0]
        y = self._proj_h(layer, h)
        Q = cfg.q_lora_rank
        q_lora = rmsnorm(y[:, :Q], lw["q_norm"], cfg.rms_eps)
        kv_raw = y[:, Q:Q + cfg.latent_dim].float()
        kv_ops.native_store(kv_raw, lw["kv_norm"], cfg.rms_eps, meta.swa_write, meta.positions, self.freqs,
                            self.pool.swa[layer])
        q_lin, qi = self._proj_q(layer, q_lora)
        q = fused_ops.rope_q(q_lin.view(B, self.heads, cfg.latent_dim), meta.positions, self.freqs)
        ratio = cfg.compress_ratios[layer]
        if ratio:
            self._compress_decode(layer, y, meta)
        if ratio == abi.C4_RATIO:
            csa_slots, csa_pos = self._index_topk(layer, q_lora, y, meta.c4_phys, meta.c4_count, self.r4max, qi)
            csa_len = meta.topk_len
            pool_native, planes = self.csa_planes(layer)
            if self.observer is not None:
                self.observer.observe_query(self, layer, q, csa_slots, csa_pos, meta)
            if self.adapter_ws is not None:
                csa_slots, pool_native, planes = self._adapter_rows(planes, csa_slots, csa_pos)
        elif ratio == abi.C128_RATIO:
            csa_slots, csa_pos, csa_len = meta.c128_slots, meta.c128_pos, meta.c128_len
            pool_native, planes = self.pool.c128_native[layer], None
        else:
            csa_slots, csa_pos, csa_len = meta.no_rows, meta.no_rows, meta.zero_len
            pool_native, planes = self.pool.swa[layer], None
        o, _ = attn_ops.sparse_mla_decode(
            q, self.pool.swa[layer], meta.swa_slots, meta.swa_len, csa_slots, csa_pos, csa_len, self.freqs,
            lw["sink"], self.scale, meta.positions_i32, csa_pool=pool_native, csa_planes=planes,
            csa_fp4=self.pool.fp4_format if ratio == abi.C4_RATIO else None)
        return self._o_proj(layer, o, B)

    def _adapter_rows(self, planes, csa_slots: torch.Tensor, csa_pos: torch.Tensor):
        """Adapter decode: selected Packed rows -> Native records in a workspace (slot b * K + k)."""
        B, K = csa_slots.shape
        n = B * K
        idx = torch.arange(n, device=self.device, dtype=torch.int64)
        flat = csa_slots.reshape(-1)
        dst = torch.where(flat >= 0, idx, torch.full_like(idx, -1))
        kv_ops.packed_to_native(planes.values, planes.bitmap, planes.scales, flat.clamp_min(0), csa_pos.reshape(-1),
                                self.freqs, self.adapter_ws, dst)
        return dst.view(B, K).int().contiguous(), self.adapter_ws, None

    def _reconstruct_visible(self, planes, phys_row: torch.Tensor, n: int, csa_slots: torch.Tensor,
                             csa_pos: torch.Tensor):
        """Prefill over a Packed layout read by reconstruction (survivor counts other than 256): the
        request's first n records -> Native records in a workspace (record r at slot r, RoPE at 4 r), and
        the selected slots remapped to it (a C4 record's RoPE position is 4 x its index)."""
        dev = self.device
        r = torch.arange(n, device=dev, dtype=torch.int64)
        src = phys_row[:n].long()
        ws = torch.zeros(-(-n // abi.RECORDS_PER_PAGE) * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
        kv_ops.packed_to_native(planes.values, planes.bitmap, planes.scales, src.clamp_min(0), r * abi.C4_RATIO,
                                self.freqs, ws, torch.where(src >= 0, r, torch.full_like(r, -1)))
        slots = torch.where(csa_slots >= 0, csa_pos // abi.C4_RATIO, torch.full_like(csa_slots, -1))
        return slots.int().contiguous(), ws, None

    def _o_proj(self, layer: int, o: torch.Tensor, B: int) -> torch.Tensor:
        cfg = self.cfg
        lw = self.W["layers"][layer]
        if self.mx is not None:  # grouped LoRA projection (one weight per group), then the output projection
            o3 = o.view(B, self.groups, cfg.heads_per_group * cfg.latent_dim).transpose(0, 1)
            o_lora = torch.empty(B, self.groups, cfg.o_lora_rank, dtype=torch.bfloat16, device=o.device)
            self._dense(layer, "wo_a", o3, out=o_lora.transpose(0, 1))
            return self._all_reduce(self._dense(layer, "wo_b", o_lora.view(B, self.groups * cfg.o_lora_rank)))
        o = o.view(B, self.groups, cfg.heads_per_group * cfg.latent_dim).transpose(0, 1)
        o_lora = torch.bmm(o, lw["wo_a"]).transpose(0, 1).reshape(B, self.groups * cfg.o_lora_rank)
        if self.ar_hook is not None:
            return self.ar_hook(o_lora, lw["wo_b"])
        return self._all_reduce(o_lora @ lw["wo_b"].T)

    def _moe_block(self, layer: int, h: torch.Tensor):
        """Routed + shared experts of the normed residual h.

        Returns the residual addends (bf16, fp32 or None): on one rank the shared expert's bf16 output
        and the routed experts' fp32 sum, added to the residual by the next fused norm; over TP/EP their
        all-reduced bf16 sum.
        """
        if self.dp:
            return self._moe_block_dp(layer, h)
        cfg = self.cfg
        lw = self.W["layers"][layer]
        fz = self.fused[layer]
        if self.mx is not None:  # MXFP8 shared expert, BF16 router gate
            g = self._dense(layer, "shared_w13", h)
            logits = h @ lw["gate"].T
        else:
            gf = h @ fz["w_ffn"].T
            g, logits = gf[:, :fz["gate"]], gf[:, fz["gate"]:]
        topk_ids, topk_w = fused_ops.route_topk(logits, lw["gate_bias"], cfg.moe_topk, cfg.routed_scaling)
        out = moe_ops.experts(h, topk_ids, topk_w, lw, self.expert_base, self.local_experts, cfg.expert_format,
                              precision=self.moe_precision)
        silu = fused_ops.silu_mul(g)
        shared = self._dense(layer, "shared_w2", silu) if self.mx is not None else silu @ lw["shared_w2"].T
        if self.comm is None or self.world == 1:
            return shared, out
        if hasattr(self.comm, "all_reduce_sum"):
            return self.comm.all_reduce_sum(out, shared), None
        return self._all_reduce((out + shared.float()).to(torch.bfloat16)), None

    def _moe_block_dp(self, layer: int, h: torch.Tensor):
        """MoE under DP attention: the shared expert and the router run on this rank's tokens; the tokens
        and their routing go to every rank (one all-gather, rows padded to the largest count), each rank's
        experts take every real row, and a reduce-scatter returns each rank the sum for its own rows."""
        cfg = self.cfg
        lw = self.W["layers"][layer]
        fz = self.fused[layer]
        counts = self.dp_counts or [h.shape[0]] * self.world
        T, Tm, H = h.shape[0], max(counts), cfg.hidden_size
        k = cfg.moe_topk
        if T:
            if self.mx is not None:
                g = self._dense(layer, "shared_w13", h)
                logits = h @ lw["gate"].T
            else:
                gf = h @ fz["w_ffn"].T
                g, logits = gf[:, :fz["gate"]], gf[:, fz["gate"]:]
            ids, w = fused_ops.route_topk(logits, lw["gate_bias"], k, cfg.routed_scaling)
            route = torch.cat((ids.int(), w.float().view(torch.int32)), 1).view(torch.bfloat16)
        send = torch.zeros(Tm, H + 4 * k, dtype=torch.bfloat16, device=h.device)
        if T:
            send[:T, :H] = h
            send[:T, H:] = route
        allr = self.comm.all_gather_rows(send)  # [world * Tm, H + 4k]
        if all(c == Tm for c in counts):
            rows = None
            real = allr
        else:
            rows = torch.cat([torch.arange(c, device=h.device) + i * Tm for i, c in enumerate(counts)])
            real = allr.index_select(0, rows)
        if real.shape[0]:
            rt = real[:, H:].contiguous().view(torch.int32)
            out = moe_ops.experts(real[:, :H].contiguous(), rt[:, :k].contiguous(),
                                  rt[:, k:].contiguous().view(torch.float32),
                                  lw, self.expert_base, self.local_experts, cfg.expert_format,
                                  precision=self.moe_precision).float()
        else:
            out = torch.zeros(0, H, dtype=torch.float32, device=h.device)
        # the partial sums are reduced in fp32, as one rank sums its experts' outputs
        if rows is None:
            full = out
        else:
            full = torch.zeros(self.world * Tm, H, dtype=torch.float32, device=h.device)
            full.index_copy_(0, rows, out)
        mine = self.comm.reduce_scatter_rows(full)[:T]
        if not T:
            return None, None
        silu = fused_ops.silu_mul(g)
        shared = self._dense(layer, "shared_w2", silu) if self.mx is not None else silu @ lw["shared_w2"].T
        return shared, mine

    def dp_idle_forward(self) -> None:
        """A forward without tokens of this rank (DP attention, another rank's prefill step): every MoE
        block's exchange, so this rank's experts serve the other ranks' tokens."""
        h = torch.zeros(0, self.cfg.hidden_size, dtype=torch.bfloat16, device=self.device)
        for layer in range(self.cfg.num_layers):
            self._moe_block_dp(layer, h)

    def _layer_norms(self, layer: int):
        lw = self.W["layers"][layer]
        return lw["attn_norm"], lw["ffn_norm"]

    # ------------------------------------------------------------------ decode
    def decode(self, tokens: torch.Tensor, positions: torch.Tensor, req_slots: torch.Tensor) -> torch.Tensor:
        """One decode step for B requests -> logits [B, vocab] (fp32).

        The residual stream is bf16; each block's output is added to it by the fused norm that
        starts the next block.
        """
        eps = self.cfg.rms_eps
        meta = self.step_meta(positions, req_slots)
        x = self.W["embed"][tokens]
        d = dfp = None
        for layer in range(self.cfg.num_layers):
            n_attn, n_ffn = self._layer_norms(layer)
            x, h = fused_ops.add_rmsnorm(x, n_attn, eps, d, dfp, inplace=True)
            a = self._attention_block(layer, h, meta)
            x, h = fused_ops.add_rmsnorm(x, n_ffn, eps, a, inplace=True)
            d, dfp = self._moe_block(layer, h)
        _, h = fused_ops.add_rmsnorm(x, self.W["final_norm"], eps, d, dfp, inplace=True)
        return (h @ self.W["lm_head"].T).float()

    # ------------------------------------------------------------------ prefill
    def prefill(self, tokens: torch.Tensor, start: int, req_slot: int, score: tuple | None = None):
        """Process prompt tokens [T] of one request at positions start..start+T-1 (pages ensured).

        Returns logits of the last token.  Attention of each prompt token uses the same kernel
        as decode with per-token row lists; SWA rows of the chunk live in a scratch Native pool.
        With `score` = (targets [n] int64, top, first): also the log-probability of targets[i] after chunk
        position first + i (the next prompt token) and, with top > 0, the top log-probabilities there:
        returns (logits, (token_logprobs [n] fp32, top_values [n, top], top_ids [n, top])).
        """
        cfg = self.cfg
        dev = self.device
        T = tokens.shape[0]
        W = cfg.window
        pos = torch.arange(start, start + T, device=dev, dtype=torch.int64)
        req = torch.full((T,), req_slot, device=dev, dtype=torch.int64)
        # scratch rows j <-> token start - (W-1) + j
        n_scr = T + W - 1
        scr_pages = (n_scr + abi.RECORDS_PER_PAGE - 1) // abi.RECORDS_PER_PAGE
        j = torch.arange(W, device=dev)
        swa_slots = (torch.arange(T, device=dev)[:, None] + j[None]).int()
        tok_of = start - (W - 1) + swa_slots.long()
        swa_slots = torch.where(tok_of >= 0, swa_slots, torch.full_like(swa_slots, -1)).contiguous()
        swa_len = torch.full((T,), W, dtype=torch.int32, device=dev)
        # the window's tokens before the chunk (host-known: no device round trip per layer)
        n_prev = min(W - 1, start)
        prev_ring = req_slot * W + torch.arange(start - n_prev, start, device=dev) % W
        prev_dst = torch.arange(W - 1 - n_prev, W - 1, device=dev)
        meta_pos = pos
        x = self.W["embed"][tokens]
        pt = self.pool.page_table[req_slot].long()
        r_all = torch.arange(self.r4max, device=dev)
        pg = pt[(r_all // abi.RECORDS_PER_PAGE).clamp(max=pt.shape[0] - 1)]
        c4_phys_row = torch.where(pg >= 0, pg * abi.RECORDS_PER_PAGE + r_all % abi.RECORDS_PER_PAGE, -1)
        ct = self.pool.c128_table[req_slot].long()
        r2 = torch.arange(self.r128max, device=dev)
        pg2 = ct[(r2 // abi.RECORDS_PER_PAGE).clamp(max=ct.shape[0] - 1)]
        c128_phys_row = torch.where(pg2 >= 0, pg2 * abi.RECORDS_PER_PAGE + r2 % abi.RECORDS_PER_PAGE, -1)
        eps = cfg.rms_eps
        d = dfp = None
        for layer in range(cfg.num_layers):
            lw = self.W["layers"][layer]
            n_attn, n_ffn = self._layer_norms(layer)
            x, h = fused_ops.add_rmsnorm(x, n_attn, eps, d, dfp, inplace=True)
            y = self._proj_h(layer, h)
            Q = cfg.q_lora_rank
            q_lora = rmsnorm(y[:, :Q], lw["q_norm"], eps)
            kv_raw = y[:, Q:Q + cfg.latent_dim].float().contiguous()
            scratch = torch.zeros(scr_pages * abi.NATIVE_PAGE_BYTES, dtype=torch.uint8, device=dev)
            if n_prev:
                recs = kv_ops.native_pool_read(self.pool.swa[layer], prev_ring)
                _native_pool_write(scratch, prev_dst, recs)
            kv_ops.native_store(kv_raw, lw["kv_norm"], eps, torch.arange(W - 1, W - 1 + T, device=dev),
                                pos, self.freqs, scratch)
            last = slice(max(0, T - W), T)
            kv_ops.native_store(kv_raw[last].contiguous(), lw["kv_norm"], eps, req_slot * W + pos[last] % W,
                                pos[last], self.freqs, self.pool.swa[layer])
            q_lin, qi = self._proj_q(layer, q_lora)
            q = fused_ops.rope_q(q_lin.view(T, self.heads, cfg.latent_dim), pos, self.freqs)
            ratio = cfg.compress_ratios[layer]
            if ratio:
                self._compress_prefill(layer, y, pos, req_slot, c4_phys_row, c128_phys_row, start)
            if ratio == abi.C4_RATIO:
                count = (pos + 1) // abi.C4_RATIO
                n_vis = int(min(self.r4max, (start + T) // abi.C4_RATIO))
                lim = max(1, n_vis)
                csa_slots, csa_pos = self._index_topk_chunked(layer, q_lora, y, c4_phys_row, count, lim, qi=qi)
                csa_len = torch.full((T,), csa_slots.shape[1], dtype=torch.int32, device=dev)
                pool_native, planes = self.csa_planes(layer)
                if planes is not None and planes.values.shape[1] != abi.PACKED_KEEP:
                    csa_slots, pool_native, planes = self._reconstruct_visible(planes, c4_phys_row, lim, csa_slots,
                                                                               csa_pos)
            elif ratio == abi.C128_RATIO:
                n128 = (pos + 1) // abi.C128_RATIO
                lim = max(1, int(min(self.r128max, (start + T) // abi.C128_RATIO)))
                rr = torch.arange(lim, device=dev)
                csa_slots = torch.where(rr[None] < n128[:, None], c128_phys_row[:lim][None].expand(T, -1),
                                        torch.full((T, lim), -1, device=dev, dtype=torch.int64)).int().contiguous()
                csa_pos = (rr * abi.C128_RATIO).int()[None].expand(T, -1).contiguous()
                csa_len = torch.full((T,), lim, dtype=torch.int32, device=dev)
                pool_native, planes = self.pool.c128_native[layer], None
            else:
                csa_slots = torch.empty((T, 0), dtype=torch.int32, device=dev)
                csa_pos = torch.empty((T, 0), dtype=torch.int32, device=dev)
                csa_len = torch.zeros(T, dtype=torch.int32, device=dev)
                pool_native, planes = self.pool.swa[layer], None
            o, _ = attn_ops.sparse_mla_decode(
                q.contiguous(), scratch, swa_slots, swa_len, csa_slots, csa_pos, csa_len, self.freqs, lw["sink"],
                self.scale, meta_pos.int(), csa_pool=pool_native, csa_planes=planes,
                csa_fp4=self.pool.fp4_format if ratio == abi.C4_RATIO else None)
            a = self._o_proj(layer, o, T)
            x, h = fused_ops.add_rmsnorm(x, n_ffn, eps, a, inplace=True)
            d, dfp = self._moe_block(layer, h)
        _, h = fused_ops.add_rmsnorm(x[-1:], self.W["final_norm"], eps, d[-1:],
                                     None if dfp is None else dfp[-1:])
        logits = (h @ self.W["lm_head"].T).float()[0]
        if score is None:
            return logits
        a = score[2]
        return logits, self._score_rows(x[a:], d[a:], None if dfp is None else dfp[a:], score[0], score[1])

    def _score_rows(self, x, d, dfp, targets: torch.Tensor, top: int, rows: int = 1024):
        """Log-probabilities of `targets` after the first len(targets) positions of a prefill chunk (final
        norm and LM head in blocks of `rows`, so full-vocabulary logits exist for one block at a time)."""
        n = targets.shape[0]
        lp = torch.empty(n, dtype=torch.float32, device=x.device)
        tv = torch.empty(n, max(top, 0), dtype=torch.float32, device=x.device)
        ti = torch.empty(n, max(top, 0), dtype=torch.int64, device=x.device)
        for a in range(0, n, rows):
            b = min(n, a + rows)
            _, h = fused_ops.add_rmsnorm(x[a:b], self.W["final_norm"], self.cfg.rms_eps, d[a:b],
                                         None if dfp is None else dfp[a:b])
            logits = (h @ self.W["lm_head"].T).float()
            lse = torch.logsumexp(logits, -1)
            lp[a:b] = logits.gather(1, targets[a:b, None].long())[:, 0] - lse
            if top > 0:
                v, i = logits.topk(top, -1)
                tv[a:b] = v - lse[:, None]
                ti[a:b] = i
        return lp, tv, ti

    def _index_topk_chunked(self, layer, q_lora, y, phys_row, count, lim, block: int | None = None, qi=None):
        """Top-k of a prefill chunk's queries, `block` queries per indexer call (default: as many as keep the
        fp32 score buffer within 32M entries, 256 .. 2048)."""
        T = q_lora.shape[0]
        if block is None:
            block = max(256, min(2048, ((32 << 20) // max(1, lim)) // 4 * 4))
        outs_s, outs_p = [], []
        for t0 in range(0, T, block):
            t1 = min(T, t0 + block)
            ph = phys_row[:lim].int()[None].expand(t1 - t0, -1)  # one row for all (the indexer shares key tiles)
            s, p = self._index_topk(layer, q_lora[t0:t1], y[t0:t1], ph, count[t0:t1], lim,
                                    None if qi is None else qi[t0:t1])
            outs_s.append(s)
            outs_p.append(p)
        return torch.cat(outs_s).contiguous(), torch.cat(outs_p).contiguous()

    def _compress_prefill(self, layer, y, pos, req_slot, c4_phys_row, c128_phys_row, start: int):
        """Sequential-equivalent pooling over the chunk; stores every record completed in it."""
        lw = self.W["layers"][layer]
        fz = self.fused[layer]
        ratio = self.cfg.compress_ratios[layer]
        L, D = self.cfg.latent_dim, self.cfg.index_dim
        slot_in = pos % ratio
        c = fz["wc_kv"]
        kv = y[:, c:c + L].float()
        gate = y[:, c + L:c + 2 * L].float() + lw["c_ape"][slot_in]
        raw, rec = _pool_chunk(self.pool.comp_state[layer], req_slot, gate, kv, pos, ratio, start)
        if ratio == abi.C4_RATIO:
            c = fz["wi_k"]
            k = y[:, c:c + D].float()
            kg = y[:, c + D:c + 2 * D].float() + lw["i_ape"][slot_in]
            kraw, _ = _pool_chunk(self.pool.index_state[layer], req_slot, kg, k, pos, ratio, start)
        if not rec.numel():
            return
        if ratio == abi.C4_RATIO:
            slots = c4_phys_row[rec.clamp(max=self.r4max - 1)]
            slots = torch.where(rec < self.r4max, slots, -1)
            self._store_c4(layer, raw, slots, rec * ratio)
            self._store_index_keys(layer, kraw, slots)
        else:
            slots = c128_phys_row[rec.clamp(max=self.r128max - 1)]
            slots = torch.where(rec < self.r128max, slots, -1)
            kv_ops.native_store(raw, lw["c_norm"], self.cfg.rms_eps, slots, rec * ratio, self.freqs,
                                self.pool.c128_native[layer])


def _pool_chunk(state: torch.Tensor, req_slot: int, gate: torch.Tensor, val: torch.Tensor, pos: torch.Tensor,
                ratio: int, p0: int):
    """Online-softmax pooling of consecutive tokens (positions p0 .. p0 + T - 1, `pos`) into groups of
    `ratio`.

    Returns (raw rows of groups completed in the chunk [G, D], their record indices [G]);
    the trailing partial group is left in `state[req_slot]`.
    """
    T, D = gate.shape
    first_group = p0 // ratio
    grp = (pos // ratio) - first_group  # [T] 0-based group ids in the chunk
    ng = (p0 + T - 1) // ratio - first_group + 1
    st = state[req_slot]
    # per-group max over tokens (and the carried state for group 0)
    gmax = torch.full((ng, D), float("-inf"), device=gate.device)
    gmax = gmax.scatter_reduce(0, grp[:, None].expand(-1, D), gate, reduce="amax")
    gmax[0] = torch.maximum(gmax[0], st[0])
    e = torch.exp(gate - gmax[grp])
    l = torch.zeros(ng, D, device=gate.device).index_add_(0, grp, e)
    acc = torch.zeros(ng, D, device=gate.device).index_add_(0, grp, e * val)
    carry = torch.exp(st[0] - gmax[0])
    l[0] = l[0] + st[1] * carry
    acc[0] = acc[0] + st[2] * carry
    last_pos = p0 + T - 1
    complete_last = (last_pos % ratio) == ratio - 1
    n_done = ng if complete_last else ng - 1
    raw = acc[:n_done] / l[:n_done]
    rec = torch.arange(first_group, first_group + n_done, device=gate.device)
    if complete_last:
        state[req_slot, 0] = float("-inf")
        state[req_slot, 1:] = 0
    else:
        state[req_slot, 0] = gmax[-1]
        state[req_slot, 1] = l[-1]
        state[req_slot, 2] = acc[-1]
    return raw.contiguous(), rec


def _native_pool_write(pool: torch.Tensor, slots: torch.Tensor, recs: torch.Tensor) -> None:
    pages = pool.view(-1, abi.NATIVE_PAGE_BYTES)
    s = slots.long()
    page, r = s // abi.RECORDS_PER_PAGE, s % abi.RECORDS_PER_PAGE
    d_idx = r[:, None] * abi.NATIVE_DATA_BYTES + torch.arange(abi.NATIVE_DATA_BYTES, device=pool.device)[None]
    s_idx = (abi.RECORDS_PER_PAGE * abi.NATIVE_DATA_BYTES + r[:, None] * abi.NATIVE_SCALE_BYTES
             + torch.arange(abi.NATIVE_SCALE_BYTES, device=pool.device)[None])
    pages[page[:, None], d_idx] = recs[:, :abi.NATIVE_DATA_BYTES]
    pages[page[:, None], s_idx] = recs[:, abi.NATIVE_DATA_BYTES:]
