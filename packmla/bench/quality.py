"""Format quality check: how far Direct (Packed 256-of-512) decoding moves the model's next-token
distribution away from Native decoding of the same model.

    python -m packmla.bench.quality --model small --prompts 8 --prompt-len 1024 --steps 64 [--device cuda]

Both engines hold the same weights (same seed).  Every prompt is prefilled in each engine, then the
same continuation (the Native engine's greedy tokens) is teacher-forced through both, one decode step
at a time, so the two runs see identical inputs and differ only in the KV format.  Per step the tool
records KL(Native || Direct) of the next-token distributions and whether the top-1 tokens agree.  It is
the serving-side counterpart of the reference's offline pruning-quality comparison (attention-output
error of the Packed read against Native, training/evaluate.py), measured at the model's output.
"""
from __future__ import annotations

import argparse
import json

import torch


def _engine(model_cfg, fmt: str, device: str, seed: int, max_context: int):
    from ..config import EngineConfig
    from ..engine.engine import Engine

    ecfg = EngineConfig(kv_cache_format=fmt, device=device, max_running_requests=1, cuda_graph_bs=[1],
                        disable_cuda_graph=True, chunked_prefill_size=8192)
    kv = None if device == "cuda" else 256 << 20
    return Engine.build(model_cfg, ecfg, device, max_context=max_context, max_requests=1, kv_bytes=kv, seed=seed)


def _prefill(eng, prompt: torch.Tensor, slot: int) -> torch.Tensor:
    chunk = eng.ecfg.chunked_prefill_size
    logits = None
    for s in range(0, prompt.numel(), chunk):
        logits = eng.model.prefill(prompt[s:s + chunk], s, slot)
    return logits.float().reshape(-1)


def format_agreement(model_cfg, prompts: list[list[int]], steps: int, device: str = "cpu", seed: int = 0) -> dict:
    dev = torch.device(device)
    max_ctx = max(len(p) for p in prompts) + steps + 8
    native, direct = (_engine(model_cfg, f, device, seed, max_ctx) for f in ("native", "direct"))
    kls, agree, first_div = [], [], []
    for p in prompts:
        toks = torch.tensor(p, dtype=torch.int64, device=dev)
        slots = [e.pool.admit(len(p) + steps + 1) for e in (native, direct)]
        ln, ld = _prefill(native, toks, slots[0]), _prefill(direct, toks, slots[1])
        div = None
        for t in range(steps):
            lpn, lpd = torch.log_softmax(ln, -1), torch.log_softmax(ld, -1)
            kls.append(float((lpn.exp() * (lpn - lpd)).sum()))
            same = int(ln.argmax()) == int(ld.argmax())
            agree.append(same)
            if not same and div is None:
                div = t
            nxt = torch.tensor([int(ln.argmax())], device=dev)  # the Native greedy token, fed to both
            pos = torch.tensor([len(p) + t], device=dev)
            ln = native.model.decode(nxt, pos, torch.tensor([slots[0]], device=dev))[0].float()
            ld = direct.model.decode(nxt, pos, torch.tensor([slots[1]], device=dev))[0].float()
        first_div.append(div)
        native.pool.release(slots[0])
        direct.pool.release(slots[1])
    k = torch.tensor(kls, dtype=torch.float64)
    return {"prompts": len(prompts), "steps": steps, "positions": len(kls),
            "kl_mean": float(k.mean()), "kl_p95": float(torch.quantile(k, 0.95)), "kl_max": float(k.max()),
            "top1_agreement": sum(agree) / len(agree), "first_divergence_step": first_div}


def main(argv=None) -> dict:
    from ..server.__main__ import model_config

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="tiny", help="tiny | small | v4-flash (random init)")
    ap.add_argument("--prompts", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--device", default="cpu", choices=["cpu", "cuda"])
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    cfg, weights = model_config(a.model)
    if weights is not None:
        raise SystemExit("the quality check builds random-init models (tiny | small | v4-flash)")
    g = torch.Generator().manual_seed(a.seed)
    prompts = [torch.randint(3, cfg.vocab_size, (a.prompt_len,), generator=g).tolist() for _ in range(a.prompts)]
    out = {"model": a.model, **format_agreement(cfg, prompts, a.steps, a.device, a.seed)}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()
