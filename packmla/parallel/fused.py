"""Fused GEMM + all-reduce and one-kernel all-reduce over NVLink peer memory.

Reference call sites (SGLang TP collectives, configured in the reference's server-info
`disable_custom_all_reduce false`, `enable_fused_moe_sum_all_reduce false`): the all-reduce after
attention's o_proj and after the MoE (routed sum + shared expert), once per layer each.  The
reference issues them as separate collectives (custom AR / NCCL ring) after the GEMM; here the
output projection's tcgen05 GEMM pushes its partial tiles to the tile owner in its epilogue, and the
MoE addends are summed and reduced in one kernel (csrc/comm_fused.cu).

`FusedComm` is a drop-in `TPComm`: `all_reduce` of other dtypes/sizes, and every call on CPU
tensors, stays on the process group.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import error_word, ext
from .comm import TPComm

NUM_SMS_B200 = 148
MAX_BPAD = 512
TILE_N = 256
AR_CHUNK_QUANTUM = 2048  # 256 threads x 8 bf16


class SymmetricBuffer:
    """One cudaMalloc'd buffer per rank, mapped by every peer through CUDA IPC handles.

    `peers` is a device int64[world] tensor of base addresses (own buffer at index `rank`); the
    kernels address a peer's copy with plain loads and stores, which NVLink carries.
    """

    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.device = device
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.nbytes = nbytes
        self.ptr, handle = ext().symm_alloc(nbytes, self.idx)
        ptrs = [self.ptr]
        self._opened: list[int] = []
        if self.world > 1:
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.ptr)
                else:
                    p = ext().symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.idx)
                    self._opened.append(p)
                    ptrs.append(p)
            dist.barrier(group=group)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)

    def close(self) -> None:
        if self.ptr is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            ext().symm_close(p, self.idx)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer still maps our buffer
        ext().symm_free(self.ptr, self.idx)
        self.ptr = None


def choose_splits(n: int, k: int, tokens: int, num_sms: int = NUM_SMS_B200, max_splits: int = 8) -> int:
    """K splits per output tile: enough CTAs to stream the weights from every SM.  Split partials are
    added on this GPU (each split CTA sums one column slice) before anything crosses NVLink, so
    splitting costs no link traffic."""
    tiles = (n // TILE_N) * -(-tokens // 128)
    best = 1
    for s in (2, 4, 8):
        if s <= max_splits and tiles * s <= num_sms and k % (64 * s) == 0 and k // s >= 256:
            best = s
    return best


def use_one_shot(world: int, nbytes: int) -> bool:
    """One hop (every rank pushes to every rank) for small messages; reduce-scatter + all-gather
    (two hops, 2 (world-1)/world of the bytes) once the (world-1)-fold push costs more link time."""
    return world <= 2 or nbytes * (world - 1) <= (2 << 20)


class FusedComm(TPComm):
    """TP communicator whose hot collectives are packmla's fused kernels."""

    def __init__(self, device: torch.device, hidden: int, group=None, max_tokens: int = MAX_BPAD,
                 max_splits: int = 8, timeout_s: float = 10.0, gemm: str = "auto", fused_max_tokens: int = 8):
        """`gemm`: "fused" runs the projection inside the all-reduce kernel (tcgen05, partial tiles pushed
        from the epilogue); "library" runs cuBLAS and then the one-kernel all-reduce; "auto" takes the
        fused kernel up to `fused_max_tokens` tokens, where it measured faster on 2 B200s (19.1 vs 21.2 us
        at 1 token; 23.2 vs 16.8 us at 16 tokens, packmla.bench.comm_bench)."""
        super().__init__(group)
        if gemm not in ("fused", "library", "auto"):
            raise ValueError("gemm must be 'fused', 'library' or 'auto'")
        self.gemm = gemm
        self.fused_max_tokens = fused_max_tokens
        if max_tokens > MAX_BPAD or hidden % TILE_N:
            raise ValueError("fused collectives support up to 512 tokens and hidden a multiple of 128")
        self.device = device
        self.hidden = hidden
        self.max_splits = max_splits
        self.max_src = self.world + max_splits  # flag slots: cross-rank partials + this GPU's split-K partials
        self.max_tiles = 256
        self.recv_elems = hidden * MAX_BPAD
        recv_bytes = 2 * self.max_src * self.recv_elems * 2  # two call parities
        gath_bytes = self.recv_elems * 2
        flag_rs = self.max_src * self.max_tiles * 4
        flag_ag = self.max_tiles * 4
        off = 0
        self.layout = []
        recv_off = off
        off += recv_bytes
        gath_off = off
        off += gath_bytes
        flag_rs_off = off
        off += flag_rs
        flag_ag_off = off
        off += flag_ag
        off = -(-off // 256) * 256
        lpart_off = off
        off += max_splits * self.recv_elems * 4
        self.layout = [recv_off, self.recv_elems, gath_off, flag_rs_off, flag_ag_off, self.max_src, self.max_tiles,
                       lpart_off]
        self.buf = SymmetricBuffer(off, device, group)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=device)
        self.err = error_word(device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.num_sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.fallbacks = 0

    def close(self) -> None:
        self.buf.close()

    # ------------------------------------------------------------------ collectives
    def gemm_all_reduce(self, x: torch.Tensor, w: torch.Tensor, splits: int | None = None,
                        one_shot: bool | None = None, prof: torch.Tensor | None = None) -> torch.Tensor:
        """sum over ranks of x @ w.T for bf16 x [B, K], w [N, K] -> bf16 [B, N] (bitwise equal on all ranks)."""
        B, K = x.shape
        N = w.shape[0]
        if (not x.is_cuda or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or B > MAX_BPAD or N % TILE_N
                or N > self.hidden or K % 64 or (N // TILE_N) * -(-B // 128) > min(self.num_sms, self.max_tiles)):
            self.fallbacks += 1
            return self.all_reduce(x @ w.T)
        library = self.gemm == "library" or (self.gemm == "auto" and B > self.fused_max_tokens)
        if library and splits is None and prof is None:
            return self.all_reduce_sum(None, x @ w.T, one_shot)
        s = splits or choose_splits(N, K, B, self.num_sms, self.max_splits)
        if one_shot is None:
            one_shot = use_one_shot(self.world, B * N * 2)
        out = torch.empty(B, N, dtype=torch.bfloat16, device=x.device)
        ext().gemm_allreduce(x.contiguous(), w.contiguous(), out, self.buf.peers, self.rank, self.world, self.layout,
                             self.epoch, self.err, s, int(one_shot), self.timeout_ns, prof)
        return out

    def all_reduce_sum(self, f: torch.Tensor | None, a: torch.Tensor | None, one_shot: bool | None = None
                       ) -> torch.Tensor:
        """sum over ranks of (f + a) for fp32 f and bf16 a of one shape -> bf16."""
        ref = f if f is not None else a
        n = ref.numel()
        if not ref.is_cuda or n % 8 or n > self.recv_elems:
            self.fallbacks += 1
            t = (f.float() if f is not None else 0) + (a.float() if a is not None else 0)
            return self.all_reduce(t.to(torch.bfloat16))
        tiles_target = min(128, self.num_sms, self.max_tiles)
        chunk = -(-n // tiles_target)
        chunk = -(-chunk // AR_CHUNK_QUANTUM) * AR_CHUNK_QUANTUM
        if one_shot is None:
            one_shot = use_one_shot(self.world, n * 2)
        out = torch.empty(ref.shape, dtype=torch.bfloat16, device=ref.device)
        ext().allreduce(None if a is None else a.contiguous(), None if f is None else f.contiguous(), out,
                        self.buf.peers, self.rank, self.world, self.layout, self.epoch, self.err, chunk,
                        int(one_shot), self.timeout_ns)
        return out

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if t.is_cuda and t.dtype == torch.bfloat16 and t.numel() % 8 == 0 and t.numel() <= self.recv_elems:
            return self.all_reduce_sum(None, t)
        return super().all_reduce(t)
