"""MoE routing and expert computation.

Routing (DeepSeek-style sigmoid scores): s = sigmoid(h G^T); the top-k of s + bias choose the
experts, their weights are s normalized over the chosen k, times `routed_scaling`.

Experts on this rank are [expert_base, expert_base + local_experts).  Tokens are replicated on
every TP/EP rank, so each rank computes its local experts' contribution and the caller's
all-reduce combines ranks (the MoE down-projection partial sums).

* MXFP4 experts on CUDA: routing lists (csrc/moe_fp4.cu), then csrc/moe_fp4_mma.cu: bulk-copy
  weight stream dequantized straight into register MMA fragments, gate/up with SiLU, down with the
  routed-weight scatter-add; weights use the fragment-ordered layout made once by
  `prepare_experts`.
* BF16 experts (tiny CPU configs, tests): PyTorch reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import error_word, ext


def route(h: torch.Tensor, gate_w: torch.Tensor, bias: torch.Tensor, topk: int, scaling: float):
    logits = (h @ gate_w.T).float()
    scores = torch.sigmoid(logits)
    _, ids = torch.topk(scores + bias, topk, dim=-1)
    w = scores.gather(1, ids)
    w = w / w.sum(-1, keepdim=True) * scaling
    return ids.int(), w


def experts_reference(h, topk_ids, topk_w, w13, w2, expert_base, local_experts):
    """BF16 experts, fp32 accumulation: sum_k w_k * W2 (silu(W1 h) * W3 h) over local experts."""
    T = h.shape[0]
    out = torch.zeros(T, w2.shape[1], dtype=torch.float32, device=h.device)
    I = w13.shape[1] // 2
    for le in range(local_experts):
        mask = topk_ids == (expert_base + le)
        tok, kk = torch.nonzero(mask, as_tuple=True)
        if tok.numel() == 0:
            continue
        x = h[tok]
        gu = (x @ w13[le].T).float()
        act = (F.silu(gu[:, :I]) * gu[:, I:]).to(torch.bfloat16)
        y = (act @ w2[le].T).float()
        out.index_add_(0, tok, y * topk_w[tok, kk][:, None])
    return out


def fp4_dequant(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """MXFP4 [..., K/2] + UE8M0 [..., K/32] -> fp32 [..., K] (reference path, any device)."""
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                       device=w.device)
    lo = lut[(w & 0xF).long()]
    hi = lut[(w >> 4).long()]
    vals = torch.stack((lo, hi), -1).flatten(-2)
    scale = torch.exp2(s.float() - 127.0).repeat_interleave(32, -1)
    return vals * scale


_FRAG_INDEX: dict = {}


def _frag_index(device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gather indices of the fragment-ordered tile (row, byte) and scale (row, block) layouts."""
    key = str(device)
    if key not in _FRAG_INDEX:
        ks, rh, mt, lane, s, bi = torch.meshgrid(torch.arange(4), torch.arange(2), torch.arange(4), torch.arange(32),
                                                 torch.arange(4), torch.arange(4), indexing="ij")
        g, q = lane // 4, lane % 4
        rows = 64 * rh + 16 * mt + g + 8 * (bi & 1)
        byts = 32 * ks + 8 * s + q + 4 * (bi >> 1)
        ks2, rh2, g2, mt2, blk, rsel = torch.meshgrid(torch.arange(4), torch.arange(2), torch.arange(8), torch.arange(4),
                                                      torch.arange(2), torch.arange(2), indexing="ij")
        srows = 64 * rh2 + 16 * mt2 + g2 + 8 * rsel
        sblk = 2 * ks2 + blk
        _FRAG_INDEX[key] = tuple(t.reshape(-1).to(device) for t in (rows, byts, srows, sblk))
    return _FRAG_INDEX[key]


def tile_fp4_frag(w: torch.Tensor, s: torch.Tensor, gate_up: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Canonical MXFP4 [E, R, K/2] + scales [E, R, K/32] -> register-fragment tiles (csrc/moe_fp4_mma.cu).

    Returns w_f [E, R/128, K/256, 16384] and s_f [E, R/128, K/256, 1024].  Row tile j of gate/up (R = 2I)
    holds gate rows [64 j, 64 j + 64) followed by up rows [I + 64 j, I + 64 j + 64); the down projection's
    row tiles are 128 consecutive rows.
    """
    E, R, Kh = w.shape
    K = Kh * 2
    if gate_up:
        I = R // 2
        w = torch.cat((w[:, :I].reshape(E, I // 64, 64, Kh), w[:, I:].reshape(E, I // 64, 64, Kh)), 2)
        s = torch.cat((s[:, :I].reshape(E, I // 64, 64, K // 32), s[:, I:].reshape(E, I // 64, 64, K // 32)), 2)
    else:
        w = w.reshape(E, R // 128, 128, Kh)
        s = s.reshape(E, R // 128, 128, K // 32)
    nrt, kt = w.shape[1], K // 256
    tiles = w.reshape(E, nrt, 128, kt, 128).permute(0, 1, 3, 2, 4).reshape(E, nrt, kt, 128 * 128)
    stiles = s.reshape(E, nrt, 128, kt, 8).permute(0, 1, 3, 2, 4).reshape(E, nrt, kt, 128 * 8)
    rows, byts, srows, sblk = _frag_index(w.device)
    w_f = tiles[..., rows * 128 + byts].contiguous()
    s_f = stiles[..., srows * 8 + sblk].contiguous()
    return w_f, s_f


def mx_weight_scales(s: torch.Tensor, gate_up: bool) -> torch.Tensor:
    """UE8M0 scales [E, R, K/32] -> [units, K/128, 256, 4] (csrc/moe_mxf4.cu): per unit's 256 weight rows
    (gate/up: the 128 gate rows of intermediate block j, then the matching 128 up rows; down: output
    rows 256 j .. 256 j + 255) and K-group, the 4 k-block scales of each row, rows contiguous."""
    E, R, KB = s.shape
    G = KB // 4
    if gate_up:
        I = R // 2
        x = s.reshape(E, 2, I // 128, 128, G, 4).permute(0, 2, 4, 1, 3, 5)  # E, j, g, tile, row, 4
    else:
        x = s.reshape(E, R // 256, 256, G, 4).permute(0, 1, 3, 2, 4)  # E, j, g, row, 4
    return x.reshape(-1, G, 256, 4).contiguous()


def mx_weight_scales_inverse(img: torch.Tensor, E: int, gate_up: bool) -> torch.Tensor:
    units, G = img.shape[0], img.shape[1]
    J = units // E
    if gate_up:
        x = img.reshape(E, J, G, 2, 128, 4).permute(0, 3, 1, 4, 2, 5)  # E, tile, j, row, g, 4
        return x.reshape(E, 2 * J * 128, G * 4)
    x = img.reshape(E, J, G, 256, 4).permute(0, 1, 3, 2, 4)
    return x.reshape(E, J * 256, G * 4)


def prepare_experts_mx(lw: dict, drop_canonical: bool = True) -> None:
    """Weight-scale images of the MXFP8-activation kernel; the packed weights are streamed as stored."""
    if "sfw13" in lw:
        return
    lw["sfw13"] = mx_weight_scales(lw["s13"], True)
    lw["sfw2"] = mx_weight_scales(lw["s2"], False)
    if drop_canonical:
        lw.pop("s13")
        lw.pop("s2")


def _scales(lw: dict, name: str) -> torch.Tensor:
    if name in lw:
        return lw[name]
    w = lw["w13" if name == "s13" else "w2"]
    return mx_weight_scales_inverse(lw["sfw13" if name == "s13" else "sfw2"], w.shape[0], name == "s13")


def mx_quant(x: torch.Tensor) -> torch.Tensor:
    """MXFP8 round trip of x [..., K] (fp32): E4M3 values with one UE8M0 scale per 32 (kernel rule)."""
    from ..formats import codec

    shp = x.shape
    xb = x.float().reshape(*shp[:-1], shp[-1] // 32, 32)
    e = codec.ue8m0_exponent(xb.abs().amax(-1))
    q = codec.e4m3_decode(codec.e4m3_encode(xb * codec.exp2_int(-e)[..., None]))
    return (q * codec.exp2_int(e)[..., None]).reshape(shp)


def experts_mx_reference(h, topk_ids, topk_w, lw, expert_base, local_experts):
    """fp32 oracle of the MXFP8-activation path: quantize h, MXFP4 GEMMs, SiLU-mul, quantize, GEMM."""
    T = h.shape[0]
    w13, w2 = lw["w13"], lw["w2"]
    s13, s2 = _scales(lw, "s13"), _scales(lw, "s2")
    out = torch.zeros(T, w2.shape[1], dtype=torch.float32, device=h.device)
    I = w13.shape[1] // 2
    hq = mx_quant(h.float())
    for le in range(local_experts):
        tok, kk = torch.nonzero(topk_ids == expert_base + le, as_tuple=True)
        if tok.numel() == 0:
            continue
        gu = hq[tok] @ fp4_dequant(w13[le], s13[le]).T
        act = mx_quant(F.silu(gu[:, :I]) * gu[:, I:])
        out.index_add_(0, tok, (act @ fp4_dequant(w2[le], s2[le]).T) * topk_w[tok, kk][:, None].float())
    return out


class MoEWorkspaceMX:
    """Routing lists, chunk table and MXFP8 operand images of csrc/moe_mxf4.cu (stable pointers)."""

    def __init__(self, max_tokens: int, topk: int, local_experts: int, hidden: int, inter: int, device):
        n = max_tokens * topk
        E = local_experts
        rows = (n + 31 * min(E, n) + 31) // 32 * 32
        i32 = dict(dtype=torch.int32, device=device)
        self.offsets = torch.zeros(E + 1, **i32)
        self.slot_token = torch.zeros(n, **i32)
        self.slot_weight = torch.zeros(n, dtype=torch.float32, device=device)
        self.active = torch.zeros(E + 1, **i32)
        self.pad = torch.zeros(E + 1, **i32)
        self.chunks = torch.zeros(n, 4, **i32)
        self.n_chunks = torch.zeros(1, **i32)
        u8 = dict(dtype=torch.uint8, device=device)
        self.xq = torch.zeros(hidden // 128, rows, 128, **u8)
        self.xs = torch.zeros(rows, hidden // 32, **u8)
        self.act_q = torch.zeros(inter // 128, rows, 128, **u8)
        self.act_s = torch.zeros(rows, inter // 32, **u8)
        self.max_tokens = max_tokens


def prepare_experts(lw: dict, drop_canonical: bool = True) -> None:
    """Add the kernel layout (w13_t, s13_t, w2_t, s2_t) to a layer's MXFP4 expert weights."""
    if "w13_f" in lw:
        return
    lw["w13_f"], lw["s13_f"] = tile_fp4_frag(lw["w13"], _scales(lw, "s13"), True)
    lw["w2_f"], lw["s2_f"] = tile_fp4_frag(lw["w2"], _scales(lw, "s2"), False)
    if drop_canonical:
        for k in ("w13", "s13", "w2", "s2", "sfw13", "sfw2"):
            lw.pop(k, None)


class MoEWorkspace:
    """Routing lists and activations with stable pointers (graph-capturable)."""

    def __init__(self, max_tokens: int, topk: int, local_experts: int, inter: int, device, hidden: int = 0):
        n = max_tokens * topk
        self.offsets = torch.zeros(local_experts + 1, dtype=torch.int32, device=device)
        self.slot_token = torch.zeros(n, dtype=torch.int32, device=device)
        self.slot_weight = torch.zeros(n, dtype=torch.float32, device=device)
        self.active = torch.zeros(local_experts + 1, dtype=torch.int32, device=device)
        rows = n + 16 * local_experts  # padded per-expert slot rows (each list starts on a multiple of 16)
        self.pad = torch.zeros(local_experts + 1, dtype=torch.int32, device=device)
        self.act = torch.zeros(rows, inter, dtype=torch.float16, device=device)  # down-pass token rows
        self.xs = torch.zeros(rows, hidden, dtype=torch.float16, device=device)  # gate/up token rows
        self.max_tokens = max_tokens


_WS: dict = {}


def experts(h, topk_ids, topk_w, lw, expert_base, local_experts, expert_format, workspace=None,
            precision: str = "default", prof: torch.Tensor | None = None):
    """Routed experts -> fp32 [T, H] (sum over this rank's experts of w_k * expert_k(h)).

    precision "default": MXFP8 activations (tcgen05 block-scaled kernel, csrc/moe_mxf4.cu);
    "bf16": BF16 activations (csrc/moe_fp4_mma.cu).  BF16 experts (tiny configs) use PyTorch.
    """
    if expert_format != "mxfp4":
        return experts_reference(h, topk_ids, topk_w, lw["w13"], lw["w2"], expert_base, local_experts)
    if precision not in ("default", "bf16"):
        raise ValueError("moe precision must be 'default' or 'bf16'")
    if not h.is_cuda:
        if precision == "default":
            return experts_mx_reference(h, topk_ids, topk_w, lw, expert_base, local_experts)
        # CPU: dequantize the touched experts (tests only)
        T = h.shape[0]
        out = torch.zeros(T, lw["w2"].shape[1], dtype=torch.float32)
        I = lw["w13"].shape[1] // 2
        s13, s2 = _scales(lw, "s13"), _scales(lw, "s2")
        for le in range(local_experts):
            tok, kk = torch.nonzero(topk_ids == expert_base + le, as_tuple=True)
            if tok.numel() == 0:
                continue
            w13 = fp4_dequant(lw["w13"][le], s13[le])
            w2 = fp4_dequant(lw["w2"][le], s2[le])
            gu = h[tok].float() @ w13.T
            act = (F.silu(gu[:, :I]) * gu[:, I:]).to(torch.bfloat16).float()
            out.index_add_(0, tok, (act @ w2.T) * topk_w[tok, kk][:, None])
        return out
    T, H = h.shape
    k = topk_ids.shape[1]
    if precision == "default":
        I = lw["w13"].shape[1] // 2
        ws = workspace
        if ws is None or not isinstance(ws, MoEWorkspaceMX):
            key = ("mx", h.device.index, T, k, local_experts, H, I)
            ws = _WS.get(key)
            if ws is None:
                ws = MoEWorkspaceMX(T, k, local_experts, H, I, h.device)
                _WS[key] = ws
        if "sfw13" not in lw:
            prepare_experts_mx(lw, drop_canonical=False)
        out = torch.empty(T, H, dtype=torch.float32, device=h.device)
        ext().moe_mxf4(h.contiguous(), topk_ids.int().contiguous(), topk_w.float().contiguous(), expert_base,
                       lw["w13"], lw["sfw13"], lw["w2"], lw["sfw2"], ws.offsets, ws.slot_token, ws.slot_weight,
                       ws.active, ws.pad, ws.chunks, ws.n_chunks, ws.xq, ws.xs, ws.act_q, ws.act_s, out,
                       error_word(h.device), prof)
        return out
    I = lw["w13_f"].shape[1] * 64 if "w13_f" in lw else lw["w13"].shape[1] // 2
    ws = workspace
    if ws is None:
        key = (h.device.index, T, k, local_experts, I)
        ws = _WS.get(key)
        if ws is None:
            ws = MoEWorkspace(T, k, local_experts, I, h.device, hidden=H)
            _WS[key] = ws
    out = torch.zeros(T, H, dtype=torch.float32, device=h.device)
    if "w13_f" not in lw:
        prepare_experts(lw, drop_canonical=False)
    ext().moe_fp4_mma(h, topk_ids, topk_w, expert_base, lw["w13_f"], lw["s13_f"], lw["w2_f"], lw["s2_f"], ws.offsets,
                      ws.slot_token, ws.slot_weight, ws.active, ws.pad, ws.xs, ws.act, out, error_word(h.device))
    return out
