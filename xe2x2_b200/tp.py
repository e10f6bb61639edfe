"""Tensor-parallel GPTQ and NVFP4 linear layers: one process per GPU.

Column-parallel layers (QKV, gate|up) keep ``N/world`` output columns of every
sub-matrix (head-aligned: rank r holds its q heads, its k heads and its v
heads) and need no exchange.  Row-parallel layers (o, down) keep ``K/world``
input rows on group boundaries, compute a partial ``[M, N]`` product and sum
the partials with an NCCL all-reduce on the GEMM's stream
(``w4_tp_linear`` / ``w4_tp_allreduce`` in include/w4.h).

The reference's tensor-parallel piece is the collective alone: an in-place
bf16 ``all_reduce(SUM)`` between ranks (parallel/tp2/bench_xccl_p2p0.py:235-251,
identity check r+1 summed; parallel/tp2/bench_host_ar.py:91-105).

The shard helpers are plain tensor slicing and work on CPU tensors too (the
sharding tests run them with gloo ranks against the CPU oracle).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from . import ops, synth


# ------------------------------------------------------------------ sharding
def _column_ranges(splits, rank: int, world: int):
    """[(start, stop)] of this rank's columns within each sub-matrix of widths ``splits``."""
    out, base = [], 0
    for n in splits:
        if n % world or (n // world) % 8:
            raise ValueError(f"sub-matrix of {n} columns does not split into {world} shards of a multiple of 8")
        w = n // world
        out.append((base + rank * w, base + (rank + 1) * w))
        base += n
    return out


def shard_columns(qweight, qzeros, scales, rank: int, world: int, splits=None):
    """Column-parallel shard of a GPTQ matrix (qweight [K/8,N], qzeros [K/gs,N/8] or None, scales [K/gs,N]).

    ``splits`` lists the widths of concatenated sub-matrices (q|k|v, gate|up);
    each is split evenly and the rank's pieces are concatenated in order.
    """
    N = qweight.shape[1]
    splits = list(splits) if splits else [N]
    if sum(splits) != N:
        raise ValueError(f"splits {splits} do not add up to N={N}")
    rng = _column_ranges(splits, rank, world)
    qw = torch.cat([qweight[:, a:b] for a, b in rng], dim=1).contiguous()
    sc = torch.cat([scales[:, a:b] for a, b in rng], dim=1).contiguous()
    qz = None if qzeros is None else torch.cat([qzeros[:, a // 8:b // 8] for a, b in rng], dim=1).contiguous()
    return qw, qz, sc


def column_slices(splits, rank: int, world: int):
    """Python slices of the full output that this rank's column shard produces, in order."""
    return [slice(a, b) for a, b in _column_ranges(splits, rank, world)]


def shard_rows(qweight, qzeros, scales, rank: int, world: int, group_size: int):
    """Row-parallel shard: K/world input rows, a whole number of groups."""
    K = qweight.shape[0] * 8
    if K % (world * group_size):
        raise ValueError(f"K={K} does not split into {world} shards of whole {group_size}-row groups")
    kr = K // world
    k0, g0 = rank * kr, rank * kr // group_size
    qw = qweight[k0 // 8:(k0 + kr) // 8].contiguous()
    sc = scales[g0:g0 + kr // group_size].contiguous()
    qz = None if qzeros is None else qzeros[g0:g0 + kr // group_size].contiguous()
    return qw, qz, sc


def row_input_slice(K: int, rank: int, world: int) -> slice:
    """Columns of the layer input that the rank's row shard consumes."""
    return slice(rank * K // world, (rank + 1) * K // world)


def _nvfp4_nk(w):
    """The [N, K/2] K-contiguous codes behind an operator-layout w ([K/2, N], stride(0) == 1)."""
    if w.dim() != 2 or w.stride(0) != 1:
        raise ValueError("w must be the [K/2, N] view of [N, K/2] memory (stride(0) == 1)")
    return w.t()


def shard_nvfp4_columns(w, scale, rank: int, world: int, splits=None):
    """Column-parallel shard of an NVFP4 matrix: codes w [K/2, N] (operator layout, stride(0)
    == 1) and block scales [K/16, N]; ``splits`` as in shard_columns.  The codes keep their
    K-contiguous memory, so the shard is again an operator-layout view."""
    N = w.shape[1]
    splits = list(splits) if splits else [N]
    if sum(splits) != N:
        raise ValueError(f"splits {splits} do not add up to N={N}")
    rng = _column_ranges(splits, rank, world)
    w_nk = _nvfp4_nk(w)
    ws = torch.cat([w_nk[a:b] for a, b in rng], dim=0).contiguous().t()
    sc = torch.cat([scale[:, a:b] for a, b in rng], dim=1).contiguous()
    return ws, sc


def shard_nvfp4_rows(w, scale, rank: int, world: int, k_multiple: int = 256):
    """Row-parallel shard of an NVFP4 matrix: K/world input rows, a multiple of ``k_multiple``
    (16 keeps whole scale blocks; 256 keeps the block-scaled tensor-core path)."""
    K = w.shape[0] * 2
    if K % (world * k_multiple):
        raise ValueError(f"K={K} does not split into {world} shards of a multiple of {k_multiple}")
    kr = K // world
    k0 = rank * kr
    ws = _nvfp4_nk(w)[:, k0 // 2:(k0 + kr) // 2].contiguous().t()
    sc = scale[k0 // 16:(k0 + kr) // 16].contiguous()
    return ws, sc


# ------------------------------------------------------------------ communicator
class TPComm:
    """An NCCL communicator held by libw4, bootstrapped over torch.distributed.

    Rank 0 creates the unique id; it reaches the other ranks through
    ``dist.broadcast_object_list`` on the default (or given) process group.
    Every wait is bounded by ``timeout_ms``: a rank that never joins or never
    reaches a collective makes the others fail with W4_ERR_TIMEOUT.
    """

    def __init__(self, rank: int, world: int, timeout_ms: int = 60000, group=None, device=None):
        import torch.distributed as dist

        self.rank, self.world, self.timeout_ms = rank, world, timeout_ms
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        buf = (ctypes.c_uint8 * L.W4_TP_UNIQUE_ID_BYTES)()
        if rank == 0:
            L.call("w4_tp_get_unique_id", ctypes.cast(buf, ctypes.c_void_p))
        obj = [bytes(buf) if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(obj, src=0, group=group)
        uid = (ctypes.c_uint8 * L.W4_TP_UNIQUE_ID_BYTES).from_buffer_copy(obj[0])
        self._h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            L.call("w4_tp_comm_init", ctypes.byref(self._h), world, rank, ctypes.cast(uid, ctypes.c_void_p),
                   timeout_ms)

    @property
    def handle(self):
        if self._h is None:
            raise RuntimeError("communicator is closed")
        return self._h

    def allreduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over ranks (f16 / bf16 / f32) on the current stream."""
        ops._need_cuda(t)
        ops._contig(t, "t")
        L.call("w4_tp_allreduce", self.handle, ops._p(t), t.numel(), ops._DT[t.dtype], ops._stream(t.device))
        return t

    def set_fused_epilogue(self, on: bool):
        """Row-parallel decode layers reduce in the GEMM's own epilogue, or run GEMM +
        all-reduce (the default; every rank must choose the same)."""
        L.call("w4_tp_set_fused_epilogue", self.handle, 1 if on else 0)

    def wait(self, timeout_ms: int | None = None):
        """Block until the current stream is done; W4Error(W4_ERR_TIMEOUT) if a peer is missing."""
        L.call("w4_tp_wait", self.handle, ops._stream(self.device), timeout_ms or self.timeout_ms)

    def close(self):
        """Orderly teardown (every rank calls it)."""
        if self._h is not None:
            h, self._h = self._h, None
            L.call("w4_tp_comm_destroy", h)

    def abort(self):
        """Teardown that does not wait for other ranks (after a failure anywhere)."""
        if self._h is not None:
            h, self._h = self._h, None
            L.call("w4_tp_comm_abort", h)


# ------------------------------------------------------------------ layers
class TPLinear:
    """One rank's shard of a GPTQ linear layer (``mode`` "column" or "row")."""

    def __init__(self, comm: TPComm | None, mode: str, qweight, qzeros, scales, group_size=128, zero_offset=1):
        if mode not in ("column", "row"):
            raise ValueError("mode must be 'column' or 'row'")
        if mode == "row" and comm is None:
            raise ValueError("a row-parallel layer needs a communicator")
        self.comm, self.mode = comm, mode
        self.qweight, self.qzeros, self.scales = qweight, qzeros, scales
        self.group_size, self.zero_offset = group_size, zero_offset
        self.K, self.N = qweight.shape[0] * 8, qweight.shape[1]

    def __call__(self, a, out_dtype=None, out=None):
        ops._need_cuda(a, self.qweight)
        ops._contig(a, "a")
        M, K = a.shape
        if K != self.K:
            raise ValueError(f"input has {K} features, the shard expects {self.K}")
        out_dtype = out_dtype or a.dtype
        c = out if out is not None else torch.empty((M, self.N), dtype=out_dtype, device=a.device)
        rs = torch.empty(M, dtype=torch.float32, device=a.device) if out_dtype == torch.float8_e4m3fn else None
        mode = L.W4_TP_ROW if self.mode == "row" else L.W4_TP_COLUMN
        need = L.lib().w4_tp_linear_workspace_bytes(mode, M, self.N, K, self.group_size, 0, ops._DT[out_dtype])
        ws, wsb = ops._WS.get(a.device, need)
        h = self.comm.handle if self.comm is not None else None
        L.call("w4_tp_linear", h, mode, ops._p(a), ops._DT[a.dtype], ops._p(self.qweight), ops._p(self.qzeros),
               ops._p(self.scales), None, ops._p(c), ops._DT[out_dtype], ops._p(rs), M, self.N, K,
               self.group_size, self.zero_offset, ops._p(ws), wsb, ops._stream(a.device))
        return (c, rs) if rs is not None else c


class TPLinearNVFP4:
    """One rank's shard of an NVFP4 linear layer (``mode`` "column" or "row"), bf16
    activations (W4A16) or NVFP4 activations (``act_mode`` W4_ACT_NVFP4 with the layer's
    ``a_global``).  Row-parallel outputs are summed in place with the communicator's
    all-reduce on the GEMM's stream (f32 / bf16 / f16 outputs)."""

    def __init__(self, comm: TPComm | None, mode: str, w, scale, global_scale, act_mode=None, a_global=None):
        if mode not in ("column", "row"):
            raise ValueError("mode must be 'column' or 'row'")
        if mode == "row" and comm is None:
            raise ValueError("a row-parallel layer needs a communicator")
        self.comm, self.mode = comm, mode
        self.w, self.scale, self.global_scale = w, scale, global_scale
        self.act_mode = L.W4_ACT_W4A16 if act_mode is None else act_mode
        self.a_global = a_global

    def __call__(self, x, out_dtype=torch.bfloat16):
        if out_dtype == torch.float8_e4m3fn:
            raise ValueError("fp8 row-scaled outputs need the full sum first: reduce in f32, then ops.rowscale_fp8")
        y = ops.nvfp4_gemm(x, self.w, self.scale, self.global_scale, out_dtype, self.act_mode, self.a_global)
        if self.mode == "row":
            self.comm.allreduce_(y)
        return y


@dataclass(frozen=True)
class Projection:
    name: str
    K: int
    N: int
    mode: str
    splits: tuple


def dense_27b_projections(hidden=5120, q_heads=40, kv_heads=8, head_dim=128, ffn=17408):
    """The four GPTQ projections of one 27B-class dense layer (attention math excluded)."""
    q, kv = q_heads * head_dim, kv_heads * head_dim
    return (Projection("qkv", hidden, q + 2 * kv, "column", (q, kv, kv)),
            Projection("o", q, hidden, "row", (hidden,)),
            Projection("gate_up", hidden, 2 * ffn, "column", (ffn, ffn)),
            Projection("down", ffn, hidden, "row", (hidden,)))


class TPLayerSet:
    """One rank's shards of a dense layer's projections, from seeded full weights.

    Every rank draws the same full matrices (seed per projection) and keeps its
    shard, so no weights cross GPUs.  ``step(x)`` runs QKV -> o -> gate|up ->
    down on activations x [M, hidden]; the inputs of o and down are this
    rank's slices of synthetic activations (attention and the MLP activation
    function are outside the measured path).
    """

    def __init__(self, comm, rank, world, device, group_size=128, seed=0, projections=None):
        self.rank, self.world, self.device = rank, world, device
        self.projs = projections or dense_27b_projections()
        self.layers = {}
        for i, p in enumerate(self.projs):
            qw, qz, sc, _ = synth.gptq_weights(p.K, p.N, group_size, asym=True, seed=seed + 101 * i, device=device)
            if p.mode == "column":
                shard = shard_columns(qw, qz, sc, rank, world, p.splits)
            else:
                shard = shard_rows(qw, qz, sc, rank, world, group_size)
            del qw, qz, sc
            # at world 1 a row-parallel shard is the whole matrix and nothing is summed
            mode = p.mode if world > 1 else "column"
            self.layers[p.name] = TPLinear(comm, mode, *shard, group_size=group_size)

    def inputs(self, M, dtype=torch.bfloat16, seed=7):
        """Activations for every projection's shard: {name: [M, K_rank]}."""
        out = {}
        for i, p in enumerate(self.projs):
            full = synth.activations(M, p.K, dtype, seed=seed + i, device=self.device)
            out[p.name] = full if p.mode == "column" else full[:, row_input_slice(p.K, self.rank, self.world)].contiguous()
        return out

    def step(self, xs: dict, outs: dict | None = None):
        res = {}
        for p in self.projs:
            res[p.name] = self.layers[p.name](xs[p.name], out=None if outs is None else outs[p.name])
        return res

    def flops(self, M):
        return sum(2 * M * p.N * p.K for p in self.projs)

    def weight_bytes_per_rank(self):
        tot = 0
        for lay in self.layers.values():
            tot += lay.qweight.numel() * 4 + lay.scales.numel() * 2 + (0 if lay.qzeros is None else lay.qzeros.numel() * 4)
        return tot

    def bytes(self, M, group_size=128):
        """Algorithmic bytes of one step of the whole (unsharded) layer: every weight once and the
        bf16 activations in and outputs out once (replicated reads across ranks not counted)."""
        tot = 0
        for p in self.projs:
            ngrp = p.K // group_size
            tot += p.K // 8 * p.N * 4 + ngrp * p.N * 2 + ngrp * p.N // 8 * 4 + M * (p.K + p.N) * 2
        return tot
