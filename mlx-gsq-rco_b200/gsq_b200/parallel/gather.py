"""Row-parallel decode and prefill with the gather fused into the kernels.

``RowParallelLinear`` can join the ranks' output slices with an NCCL
all-gather after the local kernel: one collective (about 10 us of latency at
decode sizes) per projection.  Instead, the matvec kernel sends each output
value straight into every rank's inbox over NVLink and each CTA collects its
share of the peers' values (``gsq_qmv_gather`` in ``include/gsq_b200.h``):
one kernel per projection, no collective launch.  The tiled matmul (prefill)
does the same from its epilogue (``gsq_qmm_gather``): each output tile is
stored into every rank's copy as it is written, and the ranks count each
other's delivered tiles.

A :class:`GatherRegion` is the per-call-site buffer behind both: every rank
allocates ``gsq_gather_region_bytes(rows, ntot)`` bytes (256 bytes of control
words, then ``rows x ntot`` values -- fp32, or fp16 for a matmul region made
with ``dtype=torch.float16`` -- then for fewer than 8 rows the matvec's
inbox), exports a CUDA IPC handle, and maps its peers' regions.  Every rank
must make the same sequence of calls on a region, and a region serves one
call site: its rows stay valid until any rank runs the same site again (that
call stores into every rank's copy, so it must not start on one rank before
every rank has consumed the previous rows: another gathered call in between,
or a barrier, orders them).
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from .. import _lib
from ..quant.layouts import type_id as _type_id


class _DeviceArray:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class GatherRegion:
    """One projection call site's gathered output on every rank of ``group``.

    ``y`` is this rank's copy, a ``rows x ntot`` tensor of ``dtype`` (a view
    of the region; ``gsq_qmv_gather`` fills all of it).  ``dtype`` is fp32, or
    fp16 for a matmul (prefill) region: the epilogue rounds each value to
    nearest even and half the bytes cross NVLink.  ``multicast`` places a
    region of 8 rows and more in symmetric memory behind an NVSwitch multicast
    address when every rank has one (one store per value, delivered to every
    rank by the switch, this one included).  Off by default (``GSQ_MULTICAST=1``
    turns it on): a multicast store also comes back over this GPU's own link,
    so every rank receives all of the output instead of the (P-1)/P that
    peer stores deliver; on 2 GPUs the peer stores were 20-25 us faster per
    17408 x 512 output.
    """

    def __init__(self, rows: int, ntot: int, group=None, device: torch.device | None = None,
                 multicast: bool | None = None, dtype: torch.dtype = torch.float32):
        if not dist.is_initialized():
            raise RuntimeError("GatherRegion needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("the fused gather supports 2 to 8 ranks")
        self.rows, self.ntot = int(rows), int(ntot)
        if dtype not in (torch.float32, torch.float16):
            raise ValueError("a gather region holds fp32 or fp16 values")
        if dtype != torch.float32 and self.rows < 8:
            raise ValueError("fp16 regions serve the matmul gather (8 rows and more)")
        self.dtype = dtype
        self._typestr = "<f4" if dtype == torch.float32 else "<f2"
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nbytes = lib.gsq_gather_region_bytes(self.rows, self.ntot)
        if nbytes == 0:
            raise ValueError("empty gather region")
        self.mc = None       # NVSwitch multicast address of the regions (prefill regions), if any
        self._symm = None
        self._imported = []
        if multicast is None:
            multicast = self.rows >= 8 and os.environ.get("GSQ_MULTICAST", "0") == "1"
        if multicast and self._symmetric(nbytes):
            return
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            _lib.check(lib.gsq_gather_region_alloc(nbytes, ctypes.byref(own)))
            self._own = own.value
            handle = ctypes.create_string_buffer(64)
            _lib.check(lib.gsq_ipc_export(own, handle))
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            ptrs, self._imported = [], []
            for i, h in enumerate(handles):
                if i == self.rank:
                    ptrs.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                _lib.check(lib.gsq_ipc_import(h, ctypes.byref(peer)))
                ptrs.append(peer.value)
                self._imported.append(peer.value)
        self.regions = (ctypes.c_void_p * self.world)(*ptrs)
        self.y = torch.as_tensor(_DeviceArray(self._own + 256, (self.rows, self.ntot), self._typestr),
                                 device=self.device)

    def _symmetric(self, nbytes: int) -> bool:
        """Regions in torch symmetric memory, mapped on every rank and, where
        the GPUs share an NVSwitch multicast object, behind one multicast
        address (``self.mc``) that the matmul's epilogue stores through once
        per value.  Collective: every rank takes the same path (all ranks
        must allocate, rendezvous and see a multicast address, or none uses
        it).  Returns False (nothing kept) when symmetric memory is not
        available on every rank."""
        group = self.group if self.group is not None else dist.group.WORLD

        def everyone(ok: bool) -> bool:
            t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
            return bool(t.item())

        buf = None
        try:
            import torch.distributed._symmetric_memory as symm
            with torch.cuda.device(self.device):
                buf = symm.empty(nbytes, dtype=torch.uint8, device=self.device)
                buf.zero_()
                torch.cuda.synchronize(self.device)
        except Exception:
            buf = None
        if not everyone(buf is not None):
            return False
        hdl = symm.rendezvous(buf, group)
        mc = int(getattr(hdl, "multicast_ptr", 0) or 0)
        ptrs = [int(p) for p in hdl.buffer_ptrs]
        if not everyone(mc != 0 and mc % 256 == 0 and all(p % 256 == 0 for p in ptrs)):
            return False
        dist.barrier(group=self.group)  # every rank's zero-filled region is in place
        self._symm = (buf, hdl)
        self.mc = mc
        self._own = ptrs[self.rank]
        self.regions = (ctypes.c_void_p * self.world)(*ptrs)
        self.y = torch.as_tensor(_DeviceArray(self._own + 256, (self.rows, self.ntot), self._typestr),
                                 device=self.device)
        return True

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (collective: every rank calls it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer still writes into this rank's region
        if self._symm is not None:
            self._symm, self.mc, self._own = None, None, None
            dist.barrier(group=self.group)
            return
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self._imported:
                _lib.check(lib.gsq_ipc_close(ctypes.c_void_p(p)))
            dist.barrier(group=self.group)
            _lib.check(lib.gsq_gather_region_free(ctypes.c_void_p(self._own)))
        self._own, self._imported = None, []


def quantized_matvec_gather(x: torch.Tensor, packed_shard: torch.Tensor, *, qtype: str, out_features: int,
                            in_features: int, region: GatherRegion, row0: int) -> torch.Tensor:
    """y = x @ deq(W).T for this rank's rows [row0, row0 + out_features) of a
    row-split projection, gathered: returns the region's ``rows x ntot`` fp32
    output, which holds every rank's rows once the call completes on the
    current stream."""
    tid = _type_id(qtype)
    dev = _lib.require_cuda(x, packed_shard)
    rows = x.numel() // in_features
    if rows != region.rows:
        raise ValueError(f"x has {rows} rows, the region {region.rows}")
    if region.dtype != torch.float32:
        raise ValueError("the matvec gathers into fp32 regions")
    flat = x.reshape(rows, in_features).contiguous()
    if flat.data_ptr() % 16:
        flat = flat.clone()
    pk = packed_shard.reshape(-1).contiguous()
    lib = _lib.load()
    need = lib.gsq_qmv_workspace_size(tid, out_features, in_features, rows)
    ws = _lib.workspaces.get(dev, need, "qmv")
    code = lib.gsq_qmv_gather(tid, flat.data_ptr(), _lib.DTYPE_CODES[flat.dtype], pk.data_ptr(), out_features,
                              in_features, rows, region.regions, region.world, region.rank, row0, region.ntot,
                              ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
                              _lib.stream_ptr(dev))
    _lib.check(code)
    return region.y


def quantized_matmul_gather(x: torch.Tensor, packed_shard: torch.Tensor, *, qtype: str, out_features: int,
                            in_features: int, region: GatherRegion, row0: int) -> torch.Tensor:
    """The tiled matmul (prefill) of this rank's rows [row0, row0 + out_features)
    of a row-split projection with the gather fused into its epilogue
    (``gsq_qmm_gather``): every output tile goes into every rank's region over
    NVLink as it is written.  Returns the first ``rows`` rows of the region's
    output (fp32 or fp16, the region's dtype; a region of R rows serves calls
    of up to R rows), complete once the call finishes on the current
    stream."""
    tid = _type_id(qtype)
    dev = _lib.require_cuda(x, packed_shard)
    rows = x.numel() // in_features
    if rows > region.rows:
        raise ValueError(f"x has {rows} rows, the region {region.rows}")
    flat = x.reshape(rows, in_features).contiguous()
    if flat.data_ptr() % 16:
        flat = flat.clone()
    pk = packed_shard.reshape(-1).contiguous()
    lib = _lib.load()
    xcode = _lib.DTYPE_CODES[flat.dtype]
    need = lib.gsq_qmm_workspace_size(tid, out_features, in_features, rows, xcode)
    ws = _lib.workspaces.get(dev, need, "qmm")
    wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
    ycode = _lib.DTYPE_CODES[region.dtype]
    if region.mc:  # one multicast store per value through the NVSwitch
        code = lib.gsq_qmm_gather_mc(tid, flat.data_ptr(), xcode, pk.data_ptr(), out_features, in_features, rows,
                                     region.regions, region.mc, region.world, region.rank, row0, region.ntot, ycode,
                                     wsp, wsn, _lib.stream_ptr(dev))
    else:
        code = lib.gsq_qmm_gather(tid, flat.data_ptr(), xcode, pk.data_ptr(), out_features, in_features, rows,
                                  region.regions, region.world, region.rank, row0, region.ntot, ycode, wsp, wsn,
                                  _lib.stream_ptr(dev))
    _lib.check(code)
    return region.y[:rows]
