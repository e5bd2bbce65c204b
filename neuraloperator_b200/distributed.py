"""Multi-GPU execution of the spectral block: one process per GPU, torch.distributed over NCCL.

* Batch sharding (1D / 2D configurations): samples are independent, so every rank runs its own
  slice of the batch and no collective touches the data path (``shard_batch`` / ``gather_batch``).
  This replaces DistributedDataParallel-style replication of the reference's Trainer for inference.
* 3D slab decomposition (``SlabSpectralConv``): the first spatial axis is split across ranks.  The
  kept (y, z) modes of every local x plane are exchanged with one all-to-all so that each rank holds
  whole x lines for a share of the mode blocks, transforms and contracts them, and a second
  all-to-all returns them for the local inverse planes.  Only kept modes cross NVLink (about 1.7%
  of an activation for the (32, 32, 32)-mode 256^3 configuration).  This is the data path the
  reference only sketches as an unused transpose helper (neuralop/mpu/helpers.py:81-99).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _lib, ops
from .utils import host_pipeline


def shard_batch(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's contiguous slice of the batch (the batch must divide evenly)."""
    if x.shape[0] % world:
        raise ValueError(f"batch {x.shape[0]} is not a multiple of {world} ranks")
    b = x.shape[0] // world
    return x[rank * b:(rank + 1) * b]


def gather_batch(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate every rank's slice along the batch (all_gather)."""
    world = dist.get_world_size(group)
    parts = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(parts, y_local.contiguous(), group=group)
    return torch.cat(parts, dim=0)


@dataclass
class SlabLayout:
    """Split rule of the slab decomposition (mirrors nop_spectral_slab_info).

    x planes: rank r owns [r * nx, (r + 1) * nx), nx = Nx / world.
    plane-mode blocks (8 kept (y, z) modes each, ``blocks`` in total): balanced split, the first
    ``blocks % world`` ranks take one extra.  Exchange buffers hold complex64 values; byte counts
    per peer in rank order.
    """

    rank: int
    world: int
    nx_total: int
    blocks: int
    batch: int
    in_channels: int
    out_channels: int

    @property
    def nx(self) -> int:
        return self.nx_total // self.world

    def block_count(self, r: int) -> int:
        return self.blocks // self.world + (1 if r < self.blocks % self.world else 0)

    def block_begin(self, r: int) -> int:
        return r * (self.blocks // self.world) + min(r, self.blocks % self.world)

    def _blk(self, channels: int) -> int:
        return self.batch * channels * self.nx * 8 * 8  # bytes of one block on one slab

    def send1_split(self) -> List[int]:
        return [self.block_count(s) * self._blk(self.in_channels) for s in range(self.world)]

    def recv1_split(self) -> List[int]:
        return [self.block_count(self.rank) * self._blk(self.in_channels)] * self.world

    def send2_split(self) -> List[int]:
        return [self.block_count(self.rank) * self._blk(self.out_channels)] * self.world

    def recv2_split(self) -> List[int]:
        return [self.block_count(s) * self._blk(self.out_channels) for s in range(self.world)]


class SlabSpectralConv:
    """Forward of a 3D ``SpectralConv`` whose input is split along the first spatial axis.

    ``SlabSpectralConv(conv, group)(x_slab)`` with ``x_slab`` = this rank's planes
    [B, Ci, Nx / world, Ny, Nz] returns this rank's output planes.  Weights are replicated.  The
    three compute stages run in libnop_b200 (nop_spectral_slab_*); the two exchanges are NCCL
    all-to-alls on the current stream.
    """

    def __init__(self, conv, group=None, chunks: int = 2):
        self.conv = conv
        self.group = group
        self.chunks = chunks  # batch chunks whose exchanges overlap the other chunks' transforms
        self._plans = {}
        self.exchange_events = None  # a list: (start, end) CUDA event pairs around each all-to-all

    def layout(self, x_slab: torch.Tensor, rank: Optional[int] = None, world: Optional[int] = None) -> SlabLayout:
        """Split of this rank (or of ``rank`` of ``world`` when given, without a process group)."""
        world = dist.get_world_size(self.group) if world is None else world
        rank = dist.get_rank(self.group) if rank is None else rank
        geo = self.conv.geometry([x_slab.shape[2] * world, *x_slab.shape[3:]])
        blocks = geo.kept[1] * geo.kept[2] // 8
        return SlabLayout(rank, world, x_slab.shape[2] * world, blocks, x_slab.shape[0], self.conv.in_channels,
                          self.conv.out_channels)

    # -- the three compute stages (overridable, e.g. by a host emulation in tests) --------------------
    def _plan(self, x_slab, lay: SlabLayout):
        rank, world = lay.rank, lay.world
        geo = self.conv.geometry([lay.nx_total, *x_slab.shape[3:]])
        kind, weights, ranks = self.conv.kernel_operands(geo)
        desc = ops.make_desc(geo, x_slab.shape[0], self.conv.in_channels, self.conv.out_channels,
                             weight_kind=kind, ranks=ranks, precision=self.conv.contraction_precision,
                             engine="fast")
        key = (bytes(desc), rank, world, x_slab.device.index)
        plan = self._plans.get(key)
        if plan is None:
            with torch.cuda.device(x_slab.device):
                plan = _lib.Plan(desc, slab=(rank, world))
            self._plans[key] = plan
        return plan, desc, weights

    def _packed(self, plan, desc, weights, device):
        ws = [w.detach().to(device=device, dtype=torch.complex64).contiguous() for w in weights]
        cache = self.conv.__dict__.setdefault("_nop_pack_cache", {})
        key = ("slab", bytes(desc), ops._weight_key(weights), plan.handle.value, plan.packed_bytes)
        entry = cache.get("slab_packed")
        if entry is not None and entry[0] == key:
            return entry[1]
        packed = torch.empty(plan.packed_bytes, dtype=torch.uint8, device=device)
        workspace = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=device)
        arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        _lib.check(_lib.library().nop_spectral_pack_weights(plan.handle, arr, len(ws), ctypes.c_void_p(packed.data_ptr()),
                                                            plan.packed_bytes, ctypes.c_void_p(workspace.data_ptr()),
                                                            plan.workspace_bytes, stream))
        # referenced (detached, so no autograd graph stays alive): addresses cannot be recycled
        cache["slab_packed"] = (key, packed, [w.detach() for w in weights])
        return packed

    def stage_planes_fwd(self, x_slab: torch.Tensor, lay: SlabLayout) -> torch.Tensor:
        plan, _, _ = self._plan(x_slab, lay)
        send1 = torch.empty(sum(lay.send1_split()), dtype=torch.uint8, device=x_slab.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(x_slab.device).cuda_stream)
        _lib.check(_lib.library().nop_spectral_slab_forward_planes(plan.handle, ctypes.c_void_p(x_slab.data_ptr()),
                                                                   ctypes.c_void_p(send1.data_ptr()), stream))
        return send1

    def stage_modes(self, recv1: torch.Tensor, x_slab: torch.Tensor, lay: SlabLayout) -> torch.Tensor:
        plan, desc, weights = self._plan(x_slab, lay)
        packed = self._packed(plan, desc, weights, x_slab.device)
        send2 = torch.empty(sum(lay.send2_split()), dtype=torch.uint8, device=x_slab.device)
        workspace = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=x_slab.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(x_slab.device).cuda_stream)
        _lib.check(_lib.library().nop_spectral_slab_modes(
            plan.handle, ctypes.c_void_p(recv1.data_ptr()), ctypes.c_void_p(packed.data_ptr()), plan.packed_bytes,
            ctypes.c_void_p(send2.data_ptr()), ctypes.c_void_p(workspace.data_ptr()), plan.workspace_bytes, stream))
        return send2

    def stage_planes_inv(self, recv2: torch.Tensor, x_slab: torch.Tensor, lay: SlabLayout, addend=None,
                         apply_gelu=False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        plan, _, _ = self._plan(x_slab, lay)
        shape = (x_slab.shape[0], self.conv.out_channels, *x_slab.shape[2:])
        if out is not None and (tuple(out.shape) != shape or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous tensor of shape {shape}")
        y = out if out is not None else torch.empty(shape, dtype=torch.float32, device=x_slab.device)
        b = self.conv.bias
        b = None if b is None else b.detach().reshape(-1).to(x_slab.device, torch.float32).contiguous()
        a = None if addend is None else addend.detach().to(x_slab.device, torch.float32).contiguous()
        stream = ctypes.c_void_p(torch.cuda.current_stream(x_slab.device).cuda_stream)
        _lib.check(_lib.library().nop_spectral_slab_inverse_planes(
            plan.handle, ctypes.c_void_p(recv2.data_ptr()), None if b is None else ctypes.c_void_p(b.data_ptr()),
            None if a is None else ctypes.c_void_p(a.data_ptr()), int(bool(apply_gelu)), ctypes.c_void_p(y.data_ptr()),
            stream))
        return y

    # -- one forward ------------------------------------------------------------------------------------
    def _exchange(self, recv, send, out_splits, in_splits):
        ev = self.exchange_events
        if ev is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        dist.all_to_all_single(recv, send, output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)
        if ev is not None:
            b.record()
            ev.append((a, b))

    def __call__(self, x_slab: torch.Tensor, addend: Optional[torch.Tensor] = None, apply_gelu: bool = False):
        x_slab = x_slab.contiguous()
        batch = x_slab.shape[0]
        n = self.chunks
        if self.exchange_events is None and n > 1 and batch >= n and batch % n == 0:
            return self._pipelined(x_slab, n, addend, apply_gelu)
        lay = self.layout(x_slab)
        send1 = self.stage_planes_fwd(x_slab, lay)
        recv1 = torch.empty(sum(lay.recv1_split()), dtype=send1.dtype, device=send1.device)
        self._exchange(recv1, send1, lay.recv1_split(), lay.send1_split())
        send2 = self.stage_modes(recv1, x_slab, lay)
        recv2 = torch.empty(sum(lay.recv2_split()), dtype=send2.dtype, device=send2.device)
        self._exchange(recv2, send2, lay.recv2_split(), lay.send2_split())
        return self.stage_planes_inv(recv2, x_slab, lay, addend=addend, apply_gelu=apply_gelu)

    def _pipelined(self, x_slab, n, addend, apply_gelu):
        """The forward in n batch chunks: chunk c's all-to-alls run asynchronously (NCCL's stream) while
        the current stream transforms chunk c + 1, so the exchanges overlap the plane transforms and the
        mode stage.  Every rank makes the same calls in the same order."""
        cb = x_slab.shape[0] // n
        xs = [x_slab[i * cb:(i + 1) * cb] for i in range(n)]
        lay = self.layout(xs[0])
        y = torch.empty((x_slab.shape[0], self.conv.out_channels, *x_slab.shape[2:]), dtype=torch.float32,
                        device=x_slab.device)
        keep, recv1, works = [], [], []
        for xc in xs:
            send1 = self.stage_planes_fwd(xc, lay)
            r1 = torch.empty(sum(lay.recv1_split()), dtype=send1.dtype, device=send1.device)
            works.append(dist.all_to_all_single(r1, send1, output_split_sizes=lay.recv1_split(),
                                                input_split_sizes=lay.send1_split(), group=self.group,
                                                async_op=True))
            keep.append(send1)
            recv1.append(r1)
        recv2, works2 = [], []
        for i, xc in enumerate(xs):
            works[i].wait()
            send2 = self.stage_modes(recv1[i], xc, lay)
            r2 = torch.empty(sum(lay.recv2_split()), dtype=send2.dtype, device=send2.device)
            works2.append(dist.all_to_all_single(r2, send2, output_split_sizes=lay.recv2_split(),
                                                 input_split_sizes=lay.send2_split(), group=self.group,
                                                 async_op=True))
            keep.append(send2)
            recv2.append(r2)
        for i, xc in enumerate(xs):
            works2[i].wait()
            a = None if addend is None else addend[i * cb:(i + 1) * cb]
            self.stage_planes_inv(recv2[i], xc, lay, addend=a, apply_gelu=apply_gelu, out=y[i * cb:(i + 1) * cb])
        return y

    def launches(self, x_slab: torch.Tensor) -> int:
        """Kernel launches of this library per call (the two all-to-alls are NCCL's)."""
        plan, _, _ = self._plan(x_slab, self.layout(x_slab))
        return plan.launches_per_forward


class SlabFNO:
    """Forward of a 3D ``FNO`` / ``TFNO`` whose input is split along the first spatial axis.

    ``SlabFNO(model, group)(x_slab)`` with ``x_slab`` = this rank's planes [B, Cin, Nx / world, Ny, Nz]
    returns this rank's planes of the model output.  Weights are replicated.  The lifting, the per-pixel
    part of every block and the projection are pointwise in space, so they run on the local planes (the
    grid channels placed at the slab's global x offset); every spectral layer is a ``SlabSpectralConv``
    (two NCCL all-to-alls of the kept modes).  The model must take the fused path
    (``FNO.fused_plan``); other layer shapes raise NotImplementedError.
    """

    def __init__(self, model, group=None):
        self.model = model
        self.group = group
        self.slabs = [SlabSpectralConv(conv, group) for conv in model.fno_blocks.convs]

    def _rank_world(self):
        return dist.get_rank(self.group), dist.get_world_size(self.group)

    def grid_sizes(self, x_slab: torch.Tensor):
        _, world = self._rank_world()
        return (x_slab.shape[2] * world, *x_slab.shape[3:])

    def offset(self, x_slab: torch.Tensor):
        rank, _ = self._rank_world()
        return (rank * x_slab.shape[2],) + (0,) * (x_slab.ndim - 3)

    def spectral(self, index, conv, h):
        return self.slabs[index](h)

    def instrument(self, on: bool):
        """Start (on=True) or stop recording CUDA events around every all-to-all; stopping returns the
        (start, end) pairs in call order (two per layer)."""
        if on:
            for s in self.slabs:
                s.exchange_events = []
            return None
        pairs = []
        for s in self.slabs:
            pairs += s.exchange_events or []
            s.exchange_events = None
        return pairs

    def __call__(self, x_slab: torch.Tensor) -> torch.Tensor:
        if x_slab.ndim != 5:
            raise ValueError("SlabFNO takes 3D inputs [B, C, Nx / world, Ny, Nz]")
        y = self.model.fused_forward(x_slab, spectral=self.spectral, grid_offset=self.offset(x_slab),
                                     grid_sizes=self.grid_sizes(x_slab))
        if y is None:
            raise NotImplementedError("the slab-decomposed FNO needs the fused layer shapes (FNO.fused_plan)")
        return y

    @torch.no_grad()
    def forward_host(self, x_slab: torch.Tensor, out: Optional[torch.Tensor] = None, chunk: int = 1,
                     n_streams: int = 2, synchronize: bool = True) -> torch.Tensor:
        """``__call__`` on this rank's planes held in HOST memory, cut into chunks of ``chunk`` samples whose
        copies in and out overlap the other chunks' kernels (utils.host_pipeline; ``n_streams`` is ignored).
        Every rank must make the same calls: the chunks' all-to-alls pair up in order."""
        if x_slab.is_cuda:
            raise ValueError("forward_host takes a host tensor")
        dev = next(self.model.parameters()).device
        batch = x_slab.shape[0]
        if chunk < 1 or batch % chunk:
            raise ValueError(f"chunk {chunk} does not divide the batch {batch}")
        y_shape = (batch, self.model.out_channels, *x_slab.shape[2:])
        y = out if out is not None else torch.empty(y_shape, dtype=torch.float32, pin_memory=True)
        if y.is_cuda or tuple(y.shape) != y_shape or not y.is_contiguous():
            raise ValueError(f"out must be a contiguous host tensor of shape {y_shape}")
        host_pipeline(self, x_slab, y, chunk, dev, self.__dict__.setdefault("_host_streams", {}))
        if synchronize:
            torch.cuda.current_stream(dev).synchronize()
        return y
