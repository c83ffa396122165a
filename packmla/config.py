"""Typed configuration: model geometry and engine/server options.

Model geometry of DeepSeek-V4-Flash-0731 as far as the reference records it:

* 43 served layers with MoE; compression ratio per layer [0,0,4,128,4,128,...,4]
  (server-info `_dsv4_c4_cache_compression_ratios`; MoE experts prepared for
  model.layers.0..42 in benchmarks/lswb-replay/c27-packed256-n3-20261020/kernel/repeat1/server/serve_kernel.log);
* 64 query heads over one 512-wide latent (448 NoPE + 64 RoPE), SWA window 128,
  CSA top-k 512, page 256 tokens (server-info, training/data/dataset.py:32-42);
* hidden 4096, fused q_a+kv_a output 1536 = 1024 (q LoRA) + 512 (latent), q_b
  output 16 heads x 512 per TP4 rank, o_proj input 2048 per TP4 rank, shared
  expert intermediate 2048 (DeepGEMM JIT shapes N=1536/8192/4096/1024 at K=4096/1024/2048/512
  in the same log);
* FP8 e4m3 dense weights, MXFP4 routed experts (`is_fp4_experts=True`, quant=fp8); packmla serves the
  dense projections in BF16 by default and in MXFP8 with `dense_format="fp8"`.

Values the reference does not contain (routed-expert count, top-k, vocab, indexer
width, grouped-output split) are documented assumptions sized so the weights
total ~151 GB, matching the 4 x 38.6 GB the log reports at TP4.
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field

from .formats import abi


def v4_flash_ratios(num_layers: int = 43) -> list[int]:
    ratios = []
    for i in range(num_layers):
        if i < 2:
            ratios.append(0)
        else:
            ratios.append(abi.C4_RATIO if i % 2 == 0 else abi.C128_RATIO)
    return ratios


@dataclass
class ModelConfig:
    name: str = "v4-flash"
    vocab_size: int = 129280
    hidden_size: int = 4096
    num_layers: int = 43
    num_heads: int = 64
    latent_dim: int = abi.LATENT_DIM
    rope_dim: int = abi.ROPE_DIM
    q_lora_rank: int = 1024
    o_groups: int = 8
    o_lora_rank: int = 1024
    window: int = abi.SWA_WINDOW
    compress_ratios: list[int] = field(default_factory=v4_flash_ratios)
    index_heads: int = 64
    index_dim: int = 128
    index_topk: int = 512
    n_routed_experts: int = 256
    n_shared_experts: int = 1
    moe_topk: int = 8
    moe_intermediate: int = 2048
    routed_scaling: float = 1.0
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_position: int = 1 << 20
    expert_format: str = "mxfp4"  # "mxfp4" | "bf16" (tiny CPU configs)
    # dense projections: "bf16" (cuBLAS) or "fp8" (MXFP8 weights, csrc/dense_mx.cu; the router gate and the LM
    # head stay BF16).  BF16 is the default: at decode token counts both paths are bound by per-call latency and
    # the MXFP8 kernel's is longer (measured in profiles/dense_mxfp8_projections_decode.md)
    dense_format: str = "bf16"

    def __post_init__(self):
        if len(self.compress_ratios) != self.num_layers:
            raise ValueError("compress_ratios must have one entry per layer")
        if self.num_heads % self.o_groups:
            raise ValueError("num_heads must be a multiple of o_groups")
        if self.latent_dim != abi.LATENT_DIM or self.rope_dim != abi.ROPE_DIM:
            raise ValueError("the record ABI fixes latent 512 = 448 + 64")
        if self.index_dim != 128 or self.index_heads > 64:
            raise ValueError("the indexer stores 128-wide FP8 keys and scores at most 64 heads")

    @property
    def heads_per_group(self) -> int:
        return self.num_heads // self.o_groups

    @property
    def c4_layers(self) -> list[int]:
        return [i for i, r in enumerate(self.compress_ratios) if r == abi.C4_RATIO]

    @property
    def c128_layers(self) -> list[int]:
        return [i for i, r in enumerate(self.compress_ratios) if r == abi.C128_RATIO]

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self))

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        return cls(**d)

    @classmethod
    def tiny(cls, num_layers: int = 4, **kw) -> "ModelConfig":
        """A small config with the same record ABI (latent 512) for CPU tests."""
        ratios = [0] + [abi.C4_RATIO if i % 2 == 1 else abi.C128_RATIO for i in range(1, num_layers)]
        base = dict(
            name="tiny",
            vocab_size=512,
            hidden_size=256,
            num_layers=num_layers,
            num_heads=8,
            q_lora_rank=128,
            o_groups=2,
            o_lora_rank=128,
            compress_ratios=ratios,
            index_heads=4,
            index_dim=128,
            index_topk=16,
            n_routed_experts=8,
            moe_topk=2,
            moe_intermediate=128,
            expert_format="bf16",
            dense_format="bf16",
            max_position=8192,
        )
        base.update(kw)
        return cls(**base)


# C4 cache formats: FP8 Native (584 B) and Packed (328 B) records; FP4 Native (288 B) and Packed (224 B)
# records, the V4.1 cache (E2M1 + E4M3 per 16, RoPE applied at store)
KV_FORMATS = ("native", "direct", "fp4-native", "fp4-direct")


@dataclass
class EngineConfig:
    """Serving options; flag names mirror the reference server (scripts/local/run-server.sh:55-139)."""

    kv_cache_format: str = "direct"  # native | direct | fp4-native | fp4-direct
    tp: int = 1
    ep: int = 1
    mem_fraction_static: float = 0.88
    max_running_requests: int = 256
    chunked_prefill_size: int = 8192
    # alternate prefill chunks and decode steps while both are pending (False: prefill first, as long as
    # a waiting request fits)
    prefill_decode_interleave: bool = True
    context_length: int = 1 << 20
    cuda_graph_bs: list[int] = field(default_factory=lambda: [1, 2, 4, 8, 16, 24, 32, 40, 48, 64, 96, 128])
    disable_cuda_graph: bool = False
    enable_hierarchical_cache: bool = False
    hicache_ratio: float = 2.0
    hicache_mem_layout: str = "page_first"  # page_first | layer_first
    # keep a finished request's KV on the device (its slot and pages) until the space is needed; a later
    # prompt that extends it adopts the slot and prefills only the new tokens (the reference serves with
    # SGLang's radix prefix cache on; the server turns this on unless --disable-radix-cache)
    prefix_cache: bool = False
    # with the prefix cache: requests that share a prompt prefix share its KV pages, in blocks of this many
    # tokens (packmla.kv.prefix_blocks; a multiple of 256, 0 = off).  Blocks are cached where a prefill
    # chunk ends, so they are used when the block is a multiple of chunked_prefill_size.
    prefix_block_tokens: int = 8192
    keep_count: int = abi.PACKED_KEEP
    # per-layer survivor counts of the Packed C4 layout (model layer index -> count, 64 .. 448 in steps of
    # 64; the reference's --dsv4-c4-cache-layer-keep-counts).  Fixed at start-up; a layer's values plane is
    # count bytes per record.  Counts other than 256 are read by reconstruction (decode_impl "adapter").
    layer_keep_counts: dict[int, int] | None = None
    swa_full_tokens_ratio: float = 0.1
    random_seed: int = 0
    device: str = "cuda"
    fused_collectives: bool = True
    # MoE activation precision, as the reference's --flashinfer-mxfp4-moe-precision: "default" quantizes
    # expert inputs to MXFP8 (E4M3 + UE8M0 per 32) on sm_100, "bf16" keeps them in BF16.
    moe_precision: str = "default"
    # C4 attention over Packed KV: "direct" reads the planes inside the attention kernel; "adapter"
    # first reconstructs the selected rows as Native records (the reference's Adapter mode)
    decode_impl: str = "direct"
    # DP attention (the reference server's --enable-dp-attention): each rank serves its own requests with
    # every attention head; only the routed experts are split, and every MoE block exchanges tokens
    # between the ranks (all-gather in, reduce-scatter out).  Per-rank attention work does not grow with
    # the number of ranks.
    dp_attention: bool = False

    def keep_for(self, layer: int) -> int:
        """Survivor count of a C4 layer's Packed records."""
        return (self.layer_keep_counts or {}).get(layer, self.keep_count)

    def validate(self) -> None:
        """Reject unsupported combinations before any pool allocation.

        Mirrors the reference's startup checks: Direct serving supports 256 survivors
        only, and HiCache requires the 256 layout (docs/agents/numerical-and-validation.md:13-16).
        """
        if self.kv_cache_format not in KV_FORMATS:
            raise ValueError(f"--kv-cache-format must be one of {KV_FORMATS}")
        counts = {self.keep_count, *(self.layer_keep_counts or {}).values()}
        for c in counts:
            if not (64 <= c <= 448 and c % 64 == 0):
                raise ValueError(f"survivor count {c}: 64 .. 448 in steps of 64")
        if counts != {abi.PACKED_KEEP}:
            if self.kv_cache_format != "direct":
                raise ValueError("per-layer survivor counts are a Packed (direct) layout")
            if self.decode_impl != "adapter":
                raise ValueError("direct serving supports keep_count 256 only: survivor counts other than 256 are "
                                 "read by reconstruction (decode_impl adapter)")
        if self.kv_cache_format.startswith("fp4-") and self.enable_hierarchical_cache:
            raise ValueError("the FP4 cache formats do not support HiCache")
        if self.enable_hierarchical_cache and counts != {abi.PACKED_KEEP}:
            raise ValueError("HiCache requires the 256-survivor layout")
        if not 0.0 < self.mem_fraction_static <= 0.98:
            raise ValueError("mem_fraction_static must be in (0, 0.98]")
        if self.tp < 1 or self.ep < 1:
            raise ValueError("tp and ep must be >= 1")
        if self.hicache_mem_layout not in ("page_first", "layer_first"):
            raise ValueError("--hicache-mem-layout must be page_first or layer_first")
        if self.prefix_block_tokens % 256:
            raise ValueError("prefix_block_tokens must be a multiple of 256")
        if self.hicache_ratio <= 0:
            raise ValueError("hicache_ratio must be positive")
        if self.moe_precision not in ("default", "bf16"):
            raise ValueError("moe_precision must be 'default' or 'bf16'")
        if self.decode_impl not in ("direct", "adapter"):
            raise ValueError("decode_impl must be 'direct' or 'adapter'")
        if self.decode_impl == "adapter" and self.kv_cache_format != "direct":
            raise ValueError("the adapter decode reads Packed KV: it needs kv_cache_format direct")
