"""Random-init (seeded) weights of the V4-Flash-shape model, sharded for TP/EP.

Sharding for `world` ranks (tensor parallel attention, expert parallel MoE):
  * q_b columns, sinks: heads split (num_heads / world per rank)
  * wo_a groups and wo_b input rows: output groups split (o_groups / world per rank)
  * shared expert intermediate: split; routed experts: n_routed / world per rank
  * everything else replicated (latent KV projections, compressors, indexer, norms, router)
With `dp_attention` every rank holds the whole attention block and the whole shared expert (it serves
its own requests with all heads) and only the routed experts are split.
Routed experts are MXFP4 (E2M1 nibbles, low nibble = even k, UE8M0 scale per 32 k) on GPU
configs, BF16 on tiny CPU configs.  Dense projections are BF16.

Checkpoint format: a flat dict of tensors saved with safetensors-compatible names
(`layers.{i}.{name}`); see save/load below.
"""
from __future__ import annotations

import math

import torch

from ..config import ModelConfig
from ..formats import abi

FP4_BLOCK = 32


def _normal(shape, std, gen, device, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=gen)
    return t.to(dtype)


def _unit(gen, seed, tag, idx, shape, std, device):
    gen.manual_seed(seed * 1_000_003 + tag * 977 + 7919 * idx)
    return _normal(shape, std, gen, device)


def _fp4_expert(n_exp, out_f, in_f, gen, device):
    """Random MXFP4 weights [n_exp, out_f, in_f/2] + UE8M0 scales [n_exp, out_f, in_f/32]."""
    w = torch.randint(0, 256, (n_exp, out_f, in_f // 2), dtype=torch.uint8, device=device, generator=gen)
    # E2M1 codes have std ~2.93; choose 2^e so the effective std is ~1/sqrt(in_f)
    e = round(math.log2(1.0 / math.sqrt(in_f) / 2.93))
    s = torch.randint(-1, 2, (n_exp, out_f, in_f // FP4_BLOCK), dtype=torch.int32, device=device, generator=gen)
    return w, (s + e + 127).to(torch.uint8)


def init_weights(cfg: ModelConfig, rank: int = 0, world: int = 1, device="cpu", seed: int = 0,
                 dp_attention: bool = False) -> dict:
    """Per-rank weight dict.  Replicated tensors are identical on every rank (same seed).  With
    `dp_attention` the attention block and the shared expert are whole on every rank and the routed
    experts are split over the `world` ranks."""
    if cfg.num_heads % world or cfg.o_groups % world or cfg.n_routed_experts % world or cfg.moe_intermediate % world:
        raise ValueError(f"world size {world} does not divide heads/groups/experts/intermediate")
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    H, L, Q = cfg.hidden_size, cfg.latent_dim, cfg.q_lora_rank
    a_rank, a_world = (0, 1) if dp_attention else (rank, world)  # the attention / shared-expert split
    hl, gl, el = cfg.num_heads // a_world, cfg.o_groups // a_world, cfg.n_routed_experts // world
    il = cfg.moe_intermediate // a_world
    hpg = cfg.heads_per_group
    W: dict = {}

    def rep(name_seed: int):
        g.manual_seed(seed * 1_000_003 + name_seed)

    rep(1)
    W["embed"] = _normal((cfg.vocab_size, H), 1.0, g, dev)
    W["final_norm"] = torch.ones(H, dtype=torch.float32, device=dev)
    W["lm_head"] = _normal((cfg.vocab_size, H), H ** -0.5, g, dev)
    layers = []
    for i in range(cfg.num_layers):
        base = 1000 * (i + 1)
        lw = {}
        rep(base + 1)
        lw["attn_norm"] = torch.ones(H, dtype=torch.float32, device=dev)
        lw["wqkv_a"] = _normal((Q + L, H), H ** -0.5, g, dev)
        lw["q_norm"] = torch.ones(Q, dtype=torch.float32, device=dev)
        lw["kv_norm"] = (1.0 + 0.1 * torch.randn(L, generator=g, device=dev)).float()
        # sharded tensors are generated per unit (head / group / 256-row block / expert) with a
        # seed of the unit's global index, so every TP/EP split slices the same full model
        h_lo, g_lo = a_rank * hl, a_rank * gl
        lw["wq_b"] = torch.cat([_unit(g, seed, base + 2, h, (L, Q), Q ** -0.5, dev) for h in range(h_lo, h_lo + hl)])
        rep(base + 6)
        lw["sink"] = torch.randn(cfg.num_heads, generator=g, device=dev).float()[h_lo:h_lo + hl].contiguous()
        lw["wo_a"] = torch.stack([_unit(g, seed, base + 7, j, (hpg * L, cfg.o_lora_rank), (hpg * L) ** -0.5, dev)
                                  for j in range(g_lo, g_lo + gl)])
        lw["wo_b"] = torch.cat([_unit(g, seed, base + 8, j, (H, cfg.o_lora_rank),
                                      (cfg.o_groups * cfg.o_lora_rank) ** -0.5, dev) for j in range(g_lo, g_lo + gl)], 1)
        ratio = cfg.compress_ratios[i]
        if ratio:
            rep(base + 3)
            lw["wc_kv"] = _normal((L, H), H ** -0.5, g, dev)
            lw["wc_gate"] = _normal((L, H), H ** -0.5, g, dev)
            lw["c_ape"] = (0.1 * torch.randn(ratio, L, generator=g, device=dev)).float()
            lw["c_norm"] = (1.0 + 0.1 * torch.randn(L, generator=g, device=dev)).float()
            if ratio == abi.C4_RATIO:
                d = cfg.index_dim
                lw["wi_q"] = _normal((cfg.index_heads * d, Q), Q ** -0.5, g, dev)
                lw["wi_w"] = _normal((cfg.index_heads, H), H ** -0.5, g, dev)
                lw["wi_k"] = _normal((d, H), H ** -0.5, g, dev)
                lw["wi_kgate"] = _normal((d, H), H ** -0.5, g, dev)
                lw["i_ape"] = (0.1 * torch.randn(ratio, d, generator=g, device=dev)).float()
        rep(base + 4)
        lw["ffn_norm"] = torch.ones(H, dtype=torch.float32, device=dev)
        lw["gate"] = _normal((cfg.n_routed_experts, H), H ** -0.5, g, dev)
        lw["gate_bias"] = torch.zeros(cfg.n_routed_experts, dtype=torch.float32, device=dev)
        I = cfg.moe_intermediate
        blk = min(256, I // 8)  # world sizes up to 8 split the intermediate on block boundaries
        u_lo, u_n = a_rank * il // blk, il // blk
        lw["shared_w13"] = torch.cat(
            [_unit(g, seed, base + 9, u, (blk, H), H ** -0.5, dev) for u in range(u_lo, u_lo + u_n)]
            + [_unit(g, seed, base + 10, u, (blk, H), H ** -0.5, dev) for u in range(u_lo, u_lo + u_n)])
        lw["shared_w2"] = torch.cat(
            [_unit(g, seed, base + 11, u, (H, blk), I ** -0.5, dev) for u in range(u_lo, u_lo + u_n)], 1)
        e_lo = rank * el
        if cfg.expert_format == "mxfp4":
            w13, s13, w2, s2 = [], [], [], []
            for e in range(e_lo, e_lo + el):
                g.manual_seed(seed * 1_000_003 + base * 977 + 12 + 7919 * e)
                a, b = _fp4_expert(1, 2 * I, H, g, dev)
                c, d = _fp4_expert(1, H, I, g, dev)
                w13.append(a); s13.append(b); w2.append(c); s2.append(d)
            lw["w13"], lw["s13"], lw["w2"], lw["s2"] = (torch.cat(t) for t in (w13, s13, w2, s2))
        else:
            lw["w13"] = torch.stack([_unit(g, seed, base + 12, e, (2 * I, H), H ** -0.5, dev)
                                     for e in range(e_lo, e_lo + el)])
            lw["w2"] = torch.stack([_unit(g, seed, base + 13, e, (H, I), I ** -0.5, dev)
                                    for e in range(e_lo, e_lo + el)])
        layers.append(lw)
    W["layers"] = layers
    W["meta"] = {"rank": rank, "world": world, "expert_base": rank * el, "local_experts": el,
                 "dp_attention": bool(dp_attention), "attn_world": a_world}
    return W


def flatten(W: dict) -> dict[str, torch.Tensor]:
    flat = {k: v for k, v in W.items() if torch.is_tensor(v)}
    for i, lw in enumerate(W["layers"]):
        for k, v in lw.items():
            flat[f"layers.{i}.{k}"] = v
    return flat


def unflatten(flat: dict[str, torch.Tensor], cfg: ModelConfig, meta: dict) -> dict:
    W: dict = {"layers": [dict() for _ in range(cfg.num_layers)], "meta": dict(meta)}
    for k, v in flat.items():
        if k.startswith("layers."):
            _, i, name = k.split(".", 2)
            W["layers"][int(i)][name] = v
        else:
            W[k] = v
    return W


def save_checkpoint(path: str, W: dict, cfg: ModelConfig) -> None:
    """torch.save of the flat tensor dict plus config/meta (one file per rank)."""
    torch.save({"config": cfg.to_json(), "meta": W["meta"],
                "tensors": {k: v.detach().cpu() for k, v in flatten(W).items()}}, path)


def save_safetensors(directory: str, W: dict, cfg: ModelConfig, shard_bytes: int = 4 << 30) -> list[str]:
    """Sharded safetensors checkpoint (HF layout: model-0000X-of-0000N.safetensors + an index with the
    weight map; config and rank metadata in `packmla_config.json`).  Views that share storage (the
    fused per-layer projections) are saved as independent tensors."""
    import json
    import os

    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    flat = {k: v.detach().cpu().contiguous().clone() for k, v in flatten(W).items()}
    shards: list[dict] = [{}]
    size = 0
    for k in sorted(flat):
        n = flat[k].numel() * flat[k].element_size()
        if shards[-1] and size + n > shard_bytes:
            shards.append({})
            size = 0
        shards[-1][k] = flat[k]
        size += n
    names, weight_map = [], {}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(directory, name))
        names.append(name)
        weight_map.update({k: name for k in sh})
    total = sum(v.numel() * v.element_size() for v in flat.values())
    with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    with open(os.path.join(directory, "packmla_config.json"), "w") as f:
        json.dump({"config": json.loads(cfg.to_json()), "meta": W["meta"]}, f, indent=1)
    # receipt: sha256 of every shard and of the config file, checked before the weights are used
    # (reference: its model profiles pin a revision and config hash, and receipts verify shard bytes)
    receipt = {"files": {n: _sha256(os.path.join(directory, n)) for n in names + ["packmla_config.json"]}}
    with open(os.path.join(directory, "receipt.json"), "w") as f:
        json.dump(receipt, f, indent=1)
    return names


def _sha256(path: str) -> str:
    import hashlib

    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def verify_receipt(directory: str) -> None:
    """Raise ValueError if a shard or the config differs from the checkpoint's receipt."""
    import json
    import os

    with open(os.path.join(directory, "receipt.json")) as f:
        files = json.load(f)["files"]
    for name, digest in files.items():
        path = os.path.join(directory, name)
        if not os.path.exists(path) or _sha256(path) != digest:
            raise ValueError(f"checkpoint file changed or missing: {path}")


def load_safetensors(directory: str, device="cpu", verify: bool = True) -> tuple[dict, ModelConfig]:
    """Load a sharded checkpoint; with `verify` (default) and a receipt present, every shard and the
    config are hash-checked first."""
    import json
    import os

    from safetensors.torch import load_file

    if verify and os.path.exists(os.path.join(directory, "receipt.json")):
        verify_receipt(directory)

    with open(os.path.join(directory, "model.safetensors.index.json")) as f:
        index = json.load(f)
    with open(os.path.join(directory, "packmla_config.json")) as f:
        meta = json.load(f)
    cfg = ModelConfig.from_dict(meta["config"])
    flat = {}
    for name in sorted(set(index["weight_map"].values())):
        flat.update(load_file(os.path.join(directory, name), device=str(device)))
    missing = set(index["weight_map"]) - set(flat)
    if missing:
        raise ValueError(f"checkpoint shards miss tensors: {sorted(missing)[:5]}")
    return unflatten(flat, cfg, meta["meta"]), cfg


def load_checkpoint(path: str, device="cpu") -> tuple[dict, ModelConfig]:
    import json
    import os

    if os.path.isdir(path):
        return load_safetensors(path, device)
    blob = torch.load(path, map_location="cpu", weights_only=True)  # tensors, strings and dicts only
    cfg = ModelConfig.from_dict(json.loads(blob["config"]))
    flat = {k: v.to(device) for k, v in blob["tensors"].items()}
    return unflatten(flat, cfg, blob["meta"]), cfg
