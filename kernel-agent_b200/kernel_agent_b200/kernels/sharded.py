"""Column-sharded W4A4 NVFP4 linear over the GPUs of one box (configuration 4).

The reference has no collectives: its toolkit runs one linear on one device
(``quant.py:1201-1257`` ``fp4_w4a4_linear``). Sharding is an addition in the same style:

* each rank holds the output channels ``[rank * N / g, (rank + 1) * N / g)`` of the weight;
* the NVFP4 weight's tensor scale is the WHOLE weight's (``quant.py:253-254``:
  ``amax / (6 * 448)``), so the ranks agree on the amax with one all-reduce (MAX) of a float
  before quantising their shards — the codes equal the slice of the unsharded quantisation;
* X is replicated and quantised per rank (identical codes on every rank); each rank runs its
  GEMM into ``[M, N / g]`` and the bf16 shards are all-gathered and laid out as ``[M, N]``.

Two ways to assemble the output: :func:`gather_columns` (an NCCL all-gather of the shards and
one reordering copy), or :class:`PeerOutput` (fused: every rank's GEMM epilogue writes its
tiles straight into every rank's ``[M, N]`` buffer over NVLink, through CUDA IPC mappings, so
the transfer overlaps the math and no reorder is needed; two tiny all-reduces order the
buffer's uses). Collectives go through ``torch.distributed`` (NCCL on GPUs; gloo works for
the host logic).
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from .. import _native as nat
from . import gemm
from . import quant as q


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_columns(n: int, world: int, rank: int, align: int = 128) -> slice:
    """The output channels rank ``rank`` of ``world`` owns: equal, ``align``-multiple shards
    (the block-scaled GEMM's N granularity)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if n % (world * align):
        raise ValueError(f"{n} output channels do not split into {world} shards of a multiple of {align}")
    per = n // world
    return slice(rank * per, (rank + 1) * per)


def global_amax(amax_local: torch.Tensor, group=None) -> torch.Tensor:
    """The max over ranks of each rank's NaN-keeping amax (a 0-d fp32 tensor). A NaN on any
    rank makes the result NaN (as torch's amax of the whole weight would be)."""
    world, _ = _world(group)
    a = amax_local.detach().reshape(1).float().clone()
    if world == 1:
        return a.reshape(())
    nan = torch.isnan(a).to(torch.float32)
    dist.all_reduce(nan, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(a, op=dist.ReduceOp.MAX, group=group)
    return torch.where(nan > 0, torch.full_like(a, float("nan")), a).reshape(())


def quantize_fp4_weight_shard(w_shard: torch.Tensor, group=None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """NVFP4 codes / scales / tensor scale of this rank's rows of a weight, with the tensor
    scale of the whole weight (all ranks' shards): equal to slicing ``quantize_fp4(W)``."""
    if w_shard.dim() != 2:
        raise ValueError(f"expected a 2-D weight shard [out / g, in], got shape {tuple(w_shard.shape)}")
    if w_shard.shape[1] % 16:
        raise ValueError(f"in_features {w_shard.shape[1]} is not a multiple of the nvfp4 block (16)")
    nat.require_cuda(w_shard)
    w = q._rows(q._input(w_shard))
    amax = global_amax(q._amax(w), group)
    if not math.isfinite(float(amax)):
        raise ValueError("the weight has non-finite values")
    ts = torch.empty((), dtype=torch.float32, device=w.device)
    nat.call("kab_fp4_tensor_scale", amax.data_ptr(), ts.data_ptr(), nat.stream_of(w))
    codes, scales, _ = q._fp4(w, "nvfp4", nat.KAB_FP4_WEIGHT, ts=ts)
    return codes, scales, ts


def gather_columns(local: torch.Tensor, group=None, out: torch.Tensor | None = None,
                   staging: torch.Tensor | None = None) -> torch.Tensor:
    """``[M, N / g]`` on every rank -> ``[M, N]`` (rank r's block at columns r * N / g): one
    all-gather into ``[g, M, N / g]`` then one reordering copy. ``staging`` / ``out``:
    optional preallocated buffers of those shapes."""
    world, _ = _world(group)
    if world == 1:
        return local
    m, ns = local.shape
    local = local.contiguous()
    if staging is None:
        staging = torch.empty(world, m, ns, dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(staging, local, group=group)
    else:
        dist.all_gather(list(staging.unbind(0)), local, group=group)
    if out is None:
        out = torch.empty(m, world * ns, dtype=local.dtype, device=local.device)
    out.view(m, world, ns).copy_(staging.permute(1, 0, 2))
    return out


class PeerOutput:
    """A ``[M, N]`` output buffer on every rank of ``group``, each mapped into every other
    rank's address space (CUDA IPC), for GEMM epilogues that write their column shard into all
    of them. ``peer_ptrs(col0)``: the device addresses of column ``col0`` in the other ranks'
    buffers (rank order, this rank skipped). :meth:`close` unmaps them."""

    def __init__(self, m: int, n: int, dtype: torch.dtype = torch.bfloat16, device=None, group=None):
        world, rank = _world(group)
        self.group, self.world, self.rank = group, world, rank
        self.buffer = torch.empty(m, n, dtype=dtype, device=device)
        self._bases: list[int] = []
        self._offsets: list[int] = []
        if world == 1:
            return
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_int64(0)
        nat.call("kab_ipc_handle", self.buffer.data_ptr(), handle, ctypes.byref(offset))
        mine = (bytes(handle), int(offset.value))
        everyone: list = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        for r, (h, off) in enumerate(everyone):
            if r == rank:
                continue
            base = ctypes.c_void_p(0)
            nat.call("kab_ipc_open", (ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(base))
            self._bases.append(int(base.value))
            self._offsets.append(off)
        self._sync = torch.zeros(1, dtype=torch.float32, device=self.buffer.device)

    def peer_ptrs(self, col0: int = 0) -> list[int]:
        step = self.buffer.element_size() * col0
        return [b + off + step for b, off in zip(self._bases, self._offsets)]

    def barrier(self) -> None:
        """Every rank's work on its stream up to here is done before anyone goes on (one
        1-element all-reduce on the current stream)."""
        if self.world > 1:
            dist.all_reduce(self._sync, group=self.group)

    def close(self) -> None:
        for b in self._bases:
            nat.call("kab_ipc_close", ctypes.c_void_p(b))
        self._bases, self._offsets = [], []


def fp4_w4a4_linear_sharded(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, tensor_scale,
                            bias: torch.Tensor | None = None, group=None, *, out_local: torch.Tensor | None = None,
                            out: torch.Tensor | None = None, staging: torch.Tensor | None = None,
                            peers: PeerOutput | None = None) -> torch.Tensor:
    """``fp4_w4a4_linear`` with this rank's shard of the weight (``codes [N / g, K / 2]``,
    ``scales`` its ``[N / g, K / 16]`` block scales or their swizzled flat form, the whole
    weight's ``tensor_scale``, ``bias`` this shard's ``[N / g]``): the full ``[..., N]``
    output on every rank. ``peers``: the fused path (the epilogue writes the shard into every
    rank's ``peers.buffer``, which is returned); else an all-gather of the shards."""
    nat.require_cuda(x, codes)
    k = x.shape[-1]
    if k % 16:
        raise ValueError(f"the last dimension {k} is not a multiple of the nvfp4 block (16)")
    x2 = q._rows(q._input(x))
    xq, xs, outer = q._fp4(x2, "nvfp4", nat.KAB_FP4_TOKEN, swizzle=True)
    ns = codes.shape[0]
    ws = q._swizzled(scales, ns, k // 16)
    ts = torch.as_tensor(tensor_scale, dtype=torch.float32, device=x2.device)
    odt = x.dtype if x.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
    if peers is not None:
        col0 = peers.rank * ns
        peers.barrier()  # the other ranks are done with the buffers' previous contents
        gemm.nvf4(xq, xs.view(torch.uint8), outer, codes, ws, ts, bias, out_dtype=odt,
                  out=peers.buffer[:, col0:col0 + ns], peer_out=peers.peer_ptrs(col0))
        peers.barrier()  # every rank's shard has landed in every buffer
        full = peers.buffer
    else:
        y = gemm.nvf4(xq, xs.view(torch.uint8), outer, codes, ws, ts, bias, out_dtype=odt, out=out_local)
        full = gather_columns(y, group, out=out, staging=staging)
    return full.reshape(*x.shape[:-1], full.shape[-1])
