"""Capture observer and cache builder: training states from packmla's own model.

Reference: the opt-in capture observer of the serving fork (`srt/remnant/capture.py`, hooks
`observe_raw` / `observe_attention` in the compressor and attention backend) records raw C4
latents and decode queries of a Native-format server, and `training/data/dataset.py` turns them into
training states.  Here `CaptureObserver` attaches to `V4FlashModel.observer`:

* `observe_raw(layer, raw, slots)` keeps the FP32 compressor row of every stored C4 record, keyed by
  physical record id (what the Packed writer would select from);
* `observe_query(model, layer, q, csa_slots, csa_pos, meta)` turns each targeted decode query of a
  C4 layer into a state: the selected records' raw rows and RoPE, the query, the decoded Native SWA
  rows, sink/scale, and the Native target (attention over the Native codec of the same records).

`capture_cache` drives an `Engine` in Native mode over random prompts and writes a cache
(packmla.training.data.cache) with a frozen train/development split.  Captures need no GPU: the CPU
engine runs the same model.  Command line (the counterpart of the reference's
scripts/local/capture-latent.sh, which captures from a live Native server):

    python -m packmla.training.data.capture --output cache/ --model small --issues 32 --development 8
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ...formats import abi, codec
from ..calibration import Math
from ..losses import rounded_output
from .cache import frozen_split, write_cache


def _complex_table(freqs_f32: torch.Tensor) -> torch.Tensor:
    """Model RoPE table float [P, 32, 2] (cos, sin) -> complex64 [P, 32]."""
    return torch.complex(freqs_f32[..., 0].float(), freqs_f32[..., 1].float())


def _gather_heads(t: torch.Tensor, comm) -> torch.Tensor:
    """Under tensor parallelism each rank holds the contiguous head block [rank * H/world, ...): gather
    the blocks in rank order so that every rank sees all heads (reference: its capture assembles the 64
    heads from 4 ranks).  Without a multi-rank communicator the tensor is returned as is."""
    world = getattr(comm, "world", 1)
    if world <= 1:
        return t
    import torch.distributed as dist

    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=getattr(comm, "group", None))
    return torch.cat(parts, 0)


class CaptureObserver:
    def __init__(self, layers: tuple[int, ...]):
        self.layers = set(layers)
        self.raw: dict[int, dict[int, torch.Tensor]] = {layer: {} for layer in layers}
        self.targets: dict[int, tuple[str, int]] = {}  # request slot -> (rid, position to capture)
        self.ordinals: dict[str, int] = {}
        self.states: dict[int, list[dict]] = {layer: [] for layer in layers}
        self.skipped = 0

    # ------------------------------------------------------------------ hooks
    def observe_raw(self, layer: int, raw: torch.Tensor, slots: torch.Tensor) -> None:
        if layer not in self.layers:
            return
        slots = slots.detach().long().cpu()
        rows = raw.detach().float().cpu()
        keep = (slots >= 0).nonzero()[:, 0].tolist()
        store = self.raw[layer]
        for i in keep:
            store[int(slots[i])] = rows[i].clone()

    def observe_query(self, model, layer: int, q: torch.Tensor, csa_slots: torch.Tensor, csa_pos: torch.Tensor,
                      meta) -> None:
        if layer not in self.layers or not self.targets:
            return
        req = meta.req_slots.detach().cpu().tolist()
        pos = meta.positions.detach().cpu().tolist()
        for b, (slot, p) in enumerate(zip(req, pos)):
            tgt = self.targets.get(slot)
            if tgt is None or tgt[1] != p:
                continue
            self._capture(model, layer, tgt[0], b, p, q, csa_slots, csa_pos, meta)

    # ------------------------------------------------------------------ state
    def _capture(self, model, layer, rid, b, p, q, csa_slots, csa_pos, meta) -> None:
        lw = model.W["layers"][layer]
        cfg = model.cfg
        slots = csa_slots[b].detach().long().cpu()
        if bool((slots < 0).any()) or any(int(s) not in self.raw[layer] for s in slots):
            self.skipped += 1  # only fully admitted queries (every selected record present)
            return
        table = _complex_table(model.freqs.detach().cpu())
        raw = torch.stack([self.raw[layer][int(s)] for s in slots])
        freq = table[csa_pos[b].detach().long().cpu()]
        weight = lw["c_norm"].detach().float().cpu()
        eps = float(cfg.rms_eps)
        W = int(meta.swa_len[b])
        ring = meta.swa_slots[b, :W].detach().long()
        from ...ops import kv as kv_ops

        swa = codec.native_decode(kv_ops.native_pool_read(model.pool.swa[layer], ring.to(model.device)).cpu())
        qf = _gather_heads(q[b].detach().float().cpu(), getattr(model, "comm", None))
        sink = _gather_heads(lw["sink"].detach().float().cpu(), getattr(model, "comm", None))
        scale = float(model.scale)
        query_freq = table[p]
        native = codec.native_rows(raw, weight, eps, freq)
        out = Math.attention(qf, torch.cat((swa, native)), sink, scale)[0]
        target = rounded_output(Math, out, query_freq)
        ordinal = self.ordinals.get(f"{rid}/{layer}", 0)
        self.ordinals[f"{rid}/{layer}"] = ordinal + 1
        self.states[layer].append({
            "rid": rid, "ordinal": ordinal, "layer": layer, "raw": raw.contiguous(), "freq": freq.contiguous(),
            "weight": weight.contiguous(), "eps": eps, "q": qf.contiguous(), "sink": sink.contiguous(),
            "scale": scale, "swa": swa.contiguous(), "query_freq": query_freq.contiguous(),
            "target": target.contiguous(), "reference_squared_norm": float(target.square().sum())})


def capture_cache(output: Path, model_cfg, *, issues: int = 6, development: int = 2, train_queries: int = 2,
                  dev_queries: int = 3, prompt_len: int = 300, seed: int = 0, device: str = "cpu",
                  layers: tuple[int, ...] | None = None, comm=None, publish_root: Path | None = None) -> dict:
    """Run `issues` random requests through a Native-format engine and cache their C4-layer queries.

    Each issue contributes `train_queries` (train split) or `dev_queries` (development split) decode
    positions per layer; the split is frozen by `frozen_split`.  With a multi-rank `comm` (every rank
    calls this in lockstep with the same arguments), the engine runs tensor parallel, the observer
    gathers the heads of every captured query, and rank 0 alone writes the cache.  With `publish_root`,
    rank 0 first publishes every issue's captured states there (packmla.training.data.publish) and builds
    the cache from the verified publications.
    """
    from ...config import EngineConfig
    from ...engine.engine import Engine, SamplingParams

    layers = tuple(layers) if layers is not None else tuple(model_cfg.c4_layers)
    ids = [f"issue-{i:03d}" for i in range(issues)]
    split = frozen_split(ids, development, seed)
    role_of = {rid: role for role in ("train", "development") for rid in split[role]}
    per = {"train": train_queries, "development": dev_queries}
    steps = max(train_queries, dev_queries)
    world, rank = getattr(comm, "world", 1), getattr(comm, "rank", 0)
    ecfg = EngineConfig(kv_cache_format="native", device=device, max_running_requests=2, cuda_graph_bs=[1],
                        disable_cuda_graph=True, chunked_prefill_size=8192, tp=world, ep=world)
    eng = Engine.build(model_cfg, ecfg, device, rank, world, comm if world > 1 else None,
                       max_context=prompt_len + steps + 8, max_requests=2, seed=seed)
    obs = CaptureObserver(layers)
    eng.model.observer = obs
    g = torch.Generator().manual_seed(seed)
    for rid in ids:
        prompt = torch.randint(3, model_cfg.vocab_size, (prompt_len,), generator=g).tolist()
        n_q = per[role_of[rid]]
        eng.add_request(prompt, SamplingParams(max_new_tokens=n_q + 1))
        req = eng.waiting[-1]
        while eng.has_work():
            if req.slot >= 0 and req.prefilled >= len(req.prompt):
                # the next decode step feeds position context_len - 1
                p = req.context_len - 1
                obs.targets = {req.slot: (rid, p)} if len(req.output_ids) <= n_q else {}
            eng.step()
        obs.targets = {}
    states_by_layer = {}
    for layer in layers:
        roles = {"train": [], "development": []}
        for s in obs.states[layer]:
            role = role_of[s["rid"]]
            s["role"] = role
            s["split"] = role
            roles[role].append(s)
        states_by_layer[layer] = roles
    model_info = {"name": model_cfg.name, "config": model_cfg.to_json(), "kv_cache_format": "native",
                  "capture_tp": world}
    if rank == 0 and publish_root is not None:
        from . import publish

        requests = {rid: {"split": role_of[rid]} for rid in ids}
        publish.write_capture_config(Path(publish_root), {"layers": list(layers), "split": split,
                                                          "requests": requests, "queries_captured": per,
                                                          "model": model_info})
        for rid in ids:
            publish.publish_issue(Path(publish_root), rid,
                                  {layer: [s for s in obs.states[layer] if s["rid"] == rid] for layer in layers})
        publish.build_cache(Path(publish_root), Path(output), per)
    elif rank == 0:
        write_cache(Path(output), states_by_layer, split, per, model_info)
    return {"cache": str(output), "layers": list(layers), "split": split, "skipped": obs.skipped,
            "states": {layer: {r: len(v) for r, v in roles.items()} for layer, roles in states_by_layer.items()}}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--output", type=Path, required=True, help="new cache directory")
    ap.add_argument("--model", default="tiny", help="tiny | small | v4-flash | path to a packmla checkpoint")
    ap.add_argument("--issues", type=int, default=6)
    ap.add_argument("--development", type=int, default=2)
    ap.add_argument("--train-queries", type=int, default=2)
    ap.add_argument("--dev-queries", type=int, default=3)
    ap.add_argument("--prompt-len", type=int, default=300)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--device", default="cpu", choices=["cpu", "cuda"])
    ap.add_argument("--layers", default=None, help="comma-separated C4 layers (default: all)")
    ap.add_argument("--publish", type=Path, default=None,
                    help="new publication root: publish every issue's raw captures there, build the cache from them")
    a = ap.parse_args(argv)
    if a.output.exists():
        raise SystemExit(f"{a.output} exists: captures are written to a new directory")
    from ...server.__main__ import model_config

    cfg, weights = model_config(a.model)
    if weights is not None:
        raise SystemExit("capture runs random-init models only (tiny | small | v4-flash)")
    layers = tuple(int(x) for x in a.layers.split(",")) if a.layers else None
    return capture_cache(a.output, cfg, issues=a.issues, development=a.development, train_queries=a.train_queries,
                         dev_queries=a.dev_queries, prompt_len=a.prompt_len, seed=a.seed, device=a.device,
                         layers=layers, publish_root=a.publish)


if __name__ == "__main__":
    print(json.dumps(main(), indent=2))
