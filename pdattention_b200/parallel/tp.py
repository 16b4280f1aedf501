"""Tensor parallelism for the PRA Llama-family engine (one process per GPU, NVLink peers).

Sharding (Megatron-style): the fused QKV and gate/up projections are split by output
columns (each rank owns ``H / tp`` query heads, ``Hkv / tp`` KV heads and ``F / tp``
MLP columns), the O and down projections by input rows; their partial outputs are
summed across ranks.  The chunk memory follows the heads: each rank keeps the K/V of
its own KV heads for EVERY chunk, so memory attention never moves K/V between GPUs;
the routing gists (all KV heads, ~3% of the memory) are replicated, and the routing
query slices are all-gathered, so every rank computes the same selection locally.

Collectives are this library's kernels over CUDA-IPC peer buffers
(``parallel.peer.PeerBuffers``): a one-shot all-reduce that reads every rank's
partial and fuses the residual add, and a column all-gather by peer stores.  The
row-parallel GEMM writes its partial into this rank's peer-visible buffer; the
all-reduce kernel then reads the peers' partials directly.  NCCL is used only at
set-up (gist gathering) and for host-side scalars.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _ext
from .peer import PeerBuffers


class TensorParallel:
    SMALL_ELEMS = 1 << 16  # single-buffered gathers of a few values per row (greedy sampling)
    ROUTE_K_MAX = 64       # chunks selected per row by the fused routing exchange

    def __init__(self, group=None, max_partial_elems: int = 64 << 20, max_gather_elems: int = 1 << 20,
                 max_spins: int = 1 << 23, decode_rows: int = 64, decode_width: int = 8192):
        ext = _ext.require()
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        slots = int(ext.decode_gemm_flag_slots())  # (tile, row slice) pairs of the fused decode GEMM
        self.rank = dist.get_rank(self.group)
        self.device = torch.device("cuda", torch.cuda.current_device())
        words = int(ext.tp_signal_words(self.world))
        self.max_partial = max_partial_elems
        self.max_gather = max_gather_elems
        self.buffers = PeerBuffers({
            "part0": (max_partial_elems, torch.bfloat16), "part1": (max_partial_elems, torch.bfloat16),
            "gather0": (max_gather_elems, torch.float32), "gather1": (max_gather_elems, torch.float32),
            "small": (self.SMALL_ELEMS, torch.float32),
            "dg_recv0": (self.world * decode_rows * decode_width, torch.bfloat16),
            "dg_recv1": (self.world * decode_rows * decode_width, torch.bfloat16),
            "dg_flag0": (slots * self.world, torch.int32), "dg_flag1": (slots * self.world, torch.int32),
            "route_recv": (2 * decode_rows * self.world * 2 * self.ROUTE_K_MAX, torch.float32),
            "route_flag": (decode_rows * self.world, torch.int32),
            "sig_ar": (words, torch.int32), "sig_ag": (words, torch.int32), "sig_small": (words, torch.int32)},
            self.group, self.device)
        self.parts = [self.buffers.local("part0"), self.buffers.local("part1")]
        self.part_addr = [self.buffers.addresses("part0"), self.buffers.addresses("part1")]
        self.gathers = [self.buffers.local("gather0"), self.buffers.local("gather1")]
        self.gather_addr = [self.buffers.addresses("gather0"), self.buffers.addresses("gather1")]
        self.sig_ar = self.buffers.addresses("sig_ar")
        self.sig_ag = self.buffers.addresses("sig_ag")
        self.small = self.buffers.local("small")
        self.small_addr = self.buffers.addresses("small")
        self.sig_small = self.buffers.addresses("sig_small")
        # fused GEMM + all-reduce of decode rows: two receive / flag halves, alternated per call
        self.decode_rows, self.decode_width = decode_rows, decode_width
        self.dg_recv = [self.buffers.addresses("dg_recv0"), self.buffers.addresses("dg_recv1")]
        self.dg_flags = [self.buffers.addresses("dg_flag0"), self.buffers.addresses("dg_flag1")]
        self.dg_epochs = torch.zeros(slots, dtype=torch.int32, device=self.device)
        self.epoch_dg = 0
        # fused routing exchange (local top-k pushed to every rank, merged where it lands)
        self.route_recv = self.buffers.addresses("route_recv")
        self.route_flags = self.buffers.addresses("route_flag")
        self.route_epochs = torch.zeros(decode_rows, dtype=torch.int32, device=self.device)
        self.epoch_ar = 0  # host call counters: pick the double buffer half
        self.epoch_ag = 0
        # per-CTA device call counters of the two collectives (graph-replay safe epochs)
        self.dev_epochs = torch.zeros((3, int(ext.tp_signal_words(1))), dtype=torch.int32, device=self.device)
        self.max_spins = int(max_spins)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._gist_slices: dict[int, torch.Tensor] = {}

    # -- hot path ------------------------------------------------------------------
    def gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        """``residual + sum_ranks x @ w^T`` (row-parallel projection), replicated on every rank."""
        m, n = x.shape[0], w.shape[0]
        if m * n > self.max_partial:
            raise ValueError("partial larger than the tensor-parallel buffer; lower the prefill row batch")
        half = self.epoch_ar & 1
        part = self.parts[half][: m * n].view(m, n)
        ext = _ext.require()
        ext.gemm("tn", x, w, None, part, None, None, 1.0, 0.0, None)
        out = torch.empty((m, n), device=x.device, dtype=torch.bfloat16)
        self.epoch_ar += 1
        ext.tp_allreduce(self.part_addr[half], self.sig_ar, self.rank, residual, out, self.dev_epochs[0],
                         self.max_spins, self.error)
        return out

    def fused_gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None,
                             bias: torch.Tensor | None = None, ss_out: torch.Tensor | None = None) -> torch.Tensor:
        """``residual + sum_ranks x @ w^T`` for at most ``decode_rows`` rows in ONE kernel: each
        128-feature tile's partial is pushed to every rank over NVLink as soon as it is computed
        and summed where it lands (``decode_gemm``); the row-parallel projections of decode.
        ``ss_out``: per-tile row sums of squares of the result (a folded RMSNorm after it)."""
        m, n = x.shape[0], w.shape[0]
        if m > self.decode_rows or n > self.decode_width:
            raise ValueError("fused all-reduce sized for decode rows; use gemm_allreduce")
        half = self.epoch_dg & 1
        self.epoch_dg += 1
        out = torch.empty((m, n), device=x.device, dtype=torch.bfloat16)
        _ext.require().decode_gemm(x, w, bias, residual, out, None, 0, 0, self.dg_recv[half], self.dg_flags[half],
                                   self.rank, self.dg_epochs, self.max_spins, self.error, ss_out=ss_out)
        return out

    def route_exchange(self, scores, query, gists, lo, hi, k: int, k_cand: int, budget: int, mem_max: int,
                       id_offset: int, gists_per_chunk: int, global_len, global_row0, pool_rows: int = -1):
        """This rank's exact top-k over its chunk slice, exchanged with every rank and merged in
        the same kernel (``route_topk_exchange``): ``(mem_idx, mem_len, selected ids)``, identical
        on every rank."""
        if scores.shape[0] > self.decode_rows or k > self.ROUTE_K_MAX:
            raise ValueError("routing exchange sized for decode rows and k <= 64")
        return _ext.require().route_topk_exchange(
            scores, query, gists, lo, hi, k, k_cand, budget, mem_max, id_offset, gists_per_chunk, self.route_recv,
            self.route_flags, self.route_epochs, self.rank, self.decode_rows, global_len, global_row0,
            self.max_spins, self.error, pool_rows)

    def all_gather_columns(self, x: torch.Tensor) -> torch.Tensor:
        """``[rows, cols]`` fp32 slices -> ``[rows, world * cols]`` (rank-major column blocks)."""
        rows, cols = x.shape
        if rows * cols * self.world > self.max_gather:
            raise ValueError("gather larger than the tensor-parallel buffer")
        half = self.epoch_ag & 1
        self.epoch_ag += 1
        ext = _ext.require()
        ext.tp_allgather(x.float().contiguous(), self.gather_addr[half], self.sig_ag, self.rank, self.dev_epochs[1],
                         self.max_spins, self.error)
        return self.gathers[half][: rows * cols * self.world].view(rows, cols * self.world).clone()

    def gather_small(self, x: torch.Tensor) -> torch.Tensor:
        """``[rows, cols]`` fp32 -> ``[rows, world * cols]`` through a single buffer.

        For calls separated by other collectives of this communicator (e.g. one per decode
        step, whose all-reduces keep the ranks in lockstep), so one buffer is enough and a
        captured step's double-buffer parity is untouched.  Returns a view of the buffer,
        valid until the next call."""
        rows, cols = x.shape
        if rows * cols * self.world > self.SMALL_ELEMS:
            raise ValueError("gather larger than the small tensor-parallel buffer")
        _ext.require().tp_allgather(x.float().contiguous(), self.small_addr, self.sig_small, self.rank,
                                    self.dev_epochs[2], self.max_spins, self.error)
        return self.small[: rows * cols * self.world].view(rows, cols * self.world)

    # -- memory build ---------------------------------------------------------------
    def local_gist_tables(self, mem, layer: int):
        """Tables for this rank's KV-head slice of the layer's gists (gathered later)."""
        kd = mem.kv_dim
        if layer not in self._gist_slices:
            self._gist_slices[layer] = torch.zeros((3, 1, mem.C_pad, 1, kd), device=self.device, dtype=torch.float32)
        t = self._gist_slices[layer]
        return t[1], t[2], t[0]

    def gather_gists(self, mem, first: int = 0, count: int | None = None) -> None:
        """All-gather every layer's per-slice key means of chunk slots ``first .. first + count``
        (all slots by default) and renormalise them over the full width."""
        end = mem.C_pad if count is None else first + count
        for layer, t in sorted(self._gist_slices.items()):
            local = t[1, 0, first:end, 0].contiguous()  # un-normalised key mean slice [n, kd]
            parts = [torch.empty_like(local) for _ in range(self.world)]
            dist.all_gather(parts, local, group=self.group)
            full = torch.cat(parts, dim=1)
            mem.gk[layer, first:end, 0].copy_(full)
            mem.gn[layer, first:end, 0].copy_(torch.nn.functional.normalize(full, dim=-1, eps=1e-12))
        self._gist_slices = {}

    # -- host helpers ---------------------------------------------------------------
    def max_scalar(self, value: float) -> float:
        t = torch.tensor([float(value)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def barrier(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group, device_ids=[self.device.index])

    def check(self) -> None:
        code = int(self.error.item())
        if code:
            raise RuntimeError(f"tensor-parallel collective: a peer wait timed out (phase {code - 1})")

    def close(self) -> None:
        self.check()
        self.buffers.close()
