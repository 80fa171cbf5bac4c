"""Peer-memory transport of the Fold-CP band exchange (ranks on one NVLink / NVSwitch node).

Every rank owns one window (a device buffer exported with a CUDA IPC handle, opened once by
every peer) holding two tile-sized slots. An op that reads bands of the pair plane:

  1. copies this rank's tile into slot k % 2 of its window (a snapshot, local HBM copy);
  2. passes a barrier: an all-reduce of one element over the CP group, ordered on the stream
     after the snapshot, so that no rank reads before every snapshot is complete;
  3. assembles each requested band with one ``pf_copy_regions`` launch that loads the band's
     rectangles straight out of the peers' windows over NVLink.

One barrier per op is enough because the slots alternate: a rank overwrites slot k % 2 again at
op k + 2, after the barrier of op k + 1, which no rank passes before it has finished the reads
of op k (they precede that barrier on its stream). The tile itself is never read by peers, so
the op may update it in place while peers still copy the snapshot.

This replaces the point-to-point send/receive batches and the packing/unpacking copies of the
NCCL transport (and the reference's ring exchanges, opendde/distributed/foldcp/comm.py:26-184).
Select it with ``OPENDDE_B200_FOLDCP_TRANSPORT=peer`` (the default for NCCL meshes) or fall
back to the NCCL transport with ``=nccl``.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from typing import Callable, Dict, List, Sequence, Tuple

import torch
import torch.distributed as dist

from ... import _abi, kernels
from .exchange import DistExchange, Need, Range, Region, intersect, tile_region
from .pair_sharding import FoldCPPairShardSpec

TRANSPORT_KEY = "OPENDDE_B200_FOLDCP_TRANSPORT"

# src, dst, planes, rows, row_bytes, src_pitch, dst_pitch, src_plane_pitch, dst_plane_pitch
CopyRegion = Tuple[int, int, int, int, int, int, int, int, int]


def transport_choice(backend: str) -> str:
    """The band transport of a mesh whose CP group runs on ``backend``: "peer" (the default on
    NCCL) or "nccl" (NCCL point-to-point batches) as ``OPENDDE_B200_FOLDCP_TRANSPORT`` selects;
    "dist" (torch.distributed point-to-point) for any other backend, e.g. gloo on CPU."""
    v = os.environ.get(TRANSPORT_KEY, "").strip().lower()
    if v not in ("", "peer", "nccl"):
        raise ValueError(f"{TRANSPORT_KEY} must be 'peer' or 'nccl', got {v!r}")
    if backend != "nccl":
        return "dist"
    return v or "peer"


def _slot_bytes(tile_bytes: int) -> int:
    return (tile_bytes + 255) // 256 * 256


def band_copy_plan(spec: FoldCPPairShardSpec, layout, want: Region, slot_ptrs: Sequence[int], out_ptr: int,
                   pos_bytes: int) -> List[CopyRegion]:
    """Rectangles that assemble the band ``want`` (rows x columns of the padded plane, stored
    row-major into ``out_ptr``) from every rank's tile snapshot (``slot_ptrs[q]``: rank q's
    tile, [Tr, Tc] positions of ``pos_bytes`` bytes, row-major)."""
    (nr0, nr1), (nc0, nc1) = want
    out_pitch = (nc1 - nc0) * pos_bytes
    plan: List[CopyRegion] = []
    for q in range(layout.numel):
        (tr0, tr1), (tc0, tc1) = tile_region(spec, layout.to_coord(q))
        ir, ic = intersect((tr0, tr1), (nr0, nr1)), intersect((tc0, tc1), (nc0, nc1))
        if ir is None or ic is None:
            continue
        src_pitch = (tc1 - tc0) * pos_bytes
        src = slot_ptrs[q] + (ir[0] - tr0) * src_pitch + (ic[0] - tc0) * pos_bytes
        dst = out_ptr + (ir[0] - nr0) * out_pitch + (ic[0] - nc0) * pos_bytes
        plan.append((src, dst, 1, ir[1] - ir[0], (ic[1] - ic[0]) * pos_bytes, src_pitch, out_pitch, 0, 0))
    return plan


def _round8(x: int) -> int:
    return (x + 7) // 8 * 8


def projection_geometry(spec: FoldCPPairShardSpec, coord, transposed: bool) -> Tuple[Range, Range]:
    """(rows, cols) of rank ``coord``'s tile in the projection orientation: the tile itself
    (rows R_r, cols C_c) or, transposed, (i, k) = z(k, i) (rows C_c, cols R_r)."""
    rr, cc = spec.row_range_of(coord[0]), spec.col_range_of(coord[1])
    return (cc, rr) if transposed else (rr, cc)


def projection_copy_plan(spec: FoldCPPairShardSpec, layout, rows_req: Range, transposed: bool,
                         slot_ptrs: Sequence[int], side_off: int, planes: int, elem: int, ld_t: int,
                         out_ptr: int, ld_b: int) -> List[CopyRegion]:
    """Boxes that assemble P[ch][i in rows_req][k < Np] (row pitch ld_b elements) from every
    rank's channel-major projection of its tile, P_q[ch][x][y] with x, y over the tile's rows and
    columns in the projection orientation (row pitch ld_t, at slot_ptrs[q] + side_off)."""
    i0, i1 = rows_req
    plan: List[CopyRegion] = []
    for q in range(layout.numel):
        xr, yr = projection_geometry(spec, layout.to_coord(q), transposed)
        ir = intersect(xr, rows_req)
        if ir is None or yr[1] <= yr[0]:
            continue
        nx = xr[1] - xr[0]
        src = slot_ptrs[q] + side_off + (ir[0] - xr[0]) * ld_t * elem
        dst = out_ptr + ((ir[0] - i0) * ld_b + yr[0]) * elem
        plan.append((src, dst, planes, ir[1] - ir[0], (yr[1] - yr[0]) * elem, ld_t * elem, ld_b * elem,
                     nx * ld_t * elem, (i1 - i0) * ld_b * elem))
    return plan


def _projection_side_bytes(spec: FoldCPPairShardSpec, planes: int, elem: int) -> Tuple[int, int, int]:
    """(ld_t, bytes of one side) for either orientation of a tile: the larger of the two."""
    tr, tc = spec.tile_rows, spec.tile_cols
    ld_t = _round8(max(tr, tc))
    return ld_t, _slot_bytes(planes * max(tr, tc) * ld_t * elem)


class PeerWindows:
    """This rank's IPC window and the peers' opened windows, for one CP group."""

    def __init__(self, group, cp_rank: int, numel: int, slot_bytes: int, device: torch.device) -> None:
        lib = _abi.load()
        self.group, self.cp_rank, self.numel, self.slot_bytes = group, cp_rank, numel, slot_bytes
        self.device = device
        hb = int(lib.pf_peer_handle_bytes())
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(hb)
        _abi.check(lib.pf_peer_window_alloc(2 * slot_bytes, ctypes.byref(own), handle))
        self.own = int(own.value)
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(device)
        every = torch.empty((numel, hb), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy()
        self.bases: List[int] = []
        self.opened: List[int] = []
        for q in range(numel):
            if q == cp_rank:
                self.bases.append(self.own)
                continue
            p = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(every[q].tobytes(), hb)
            _abi.check(lib.pf_peer_window_open(buf, ctypes.byref(p)))
            self.bases.append(int(p.value))
            self.opened.append(int(p.value))
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        self.slot = 0

    def slot_ptrs(self, slot: int) -> List[int]:
        return [b + slot * self.slot_bytes for b in self.bases]

    def is_remote(self, ptr: int) -> bool:
        """Whether ``ptr`` lies in a peer's window (its bytes cross NVLink when loaded)."""
        span = 2 * self.slot_bytes
        return any(b <= ptr < b + span for q, b in enumerate(self.bases) if q != self.cp_rank)

    def barrier(self) -> None:
        """Stream-ordered: work enqueued after it runs once every rank has enqueued and
        completed the work before its own barrier."""
        dist.all_reduce(self.flag, group=self.group)

    def release(self) -> None:
        """Unmap the peers' windows and free this rank's (collective: no rank reads after)."""
        lib = _abi.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            _abi.check(lib.pf_peer_window_close(ctypes.c_void_p(p)))
        self.opened = []
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        _abi.check(lib.pf_peer_window_free(ctypes.c_void_p(self.own)))
        self.own = 0


# Keyed by the CP process group and this rank's place in it. The key holds the group object
# itself, so a group that is still cached is never collected and its identity never reused by a
# new group; a new mesh over the same group reuses the same windows.
_WINDOWS: Dict[tuple, PeerWindows] = {}

# Bytes the band copies moved since the last reset, split by where their source lives: in a
# peer's window (read over NVLink) or in this GPU's memory (the tile snapshots, own bands).
COPY_BYTES = {"remote": 0, "local": 0}


def reset_copy_bytes() -> Dict[str, int]:
    out = dict(COPY_BYTES)
    COPY_BYTES["remote"] = COPY_BYTES["local"] = 0
    return out


def _window_key(mesh) -> tuple:
    return (mesh.group_2d, mesh.cp_rank)


def windows_for(mesh, slot_bytes: int, device: torch.device) -> PeerWindows:
    """The mesh's cached windows with slots of at least ``slot_bytes``, grown (collectively:
    every rank asks for the same size at the same op) when a larger request arrives."""
    need = _slot_bytes(slot_bytes)
    key = _window_key(mesh)
    w = _WINDOWS.get(key)
    if w is not None and w.slot_bytes >= need and w.device == device:
        return w
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("Fold-CP peer windows must be allocated before CUDA graph capture: run one "
                           "eager step of the same shapes first")
    if w is not None:
        w.release()
    w = PeerWindows(mesh.group_2d, mesh.cp_rank, mesh.layout.numel, need, device)
    _WINDOWS[key] = w
    return w


COPY_KEY = "OPENDDE_B200_FOLDCP_COPY"


def copy_engine() -> str:
    """Who moves the band bytes: ``"sm"`` (the pf_copy_regions kernel, default) or ``"dma"``
    (the GPU's copy engines, pf_copy_regions_dma: no SMs, so a side-stream band copy runs beside
    the persistent kernels)."""
    v = os.environ.get(COPY_KEY, "sm").strip().lower() or "sm"
    if v not in ("sm", "dma"):
        raise ValueError(f"{COPY_KEY} must be 'sm' or 'dma', got {v!r}")
    return v


RESERVE_KEY = "OPENDDE_B200_FOLDCP_RESERVE_SMS"


def reserve_sms() -> int:
    """SMs the overlapped band exchanges leave to the band-copy kernel while a chunk computes
    (``OPENDDE_B200_FOLDCP_RESERVE_SMS``, default 0). The persistent kernels otherwise hold every
    SM, and a copy kernel launched beside them waits for their end."""
    v = os.environ.get(RESERVE_KEY, "").strip()
    n = int(v) if v else 0
    if not 0 <= n <= 64:
        raise ValueError(f"{RESERVE_KEY} must be in [0, 64], got {v!r}")
    return n


@contextlib.contextmanager
def sm_reserve(n: int):
    """Launches inside use ``n`` fewer SMs for their persistent grids (the library's
    PF_OPT_SM_RESERVE on this thread); nothing changes for n = 0."""
    if n <= 0:
        yield
        return
    _abi.set_sm_reserve(n)
    try:
        yield
    finally:
        _abi.set_sm_reserve(0)


def peer_copy_gbs(mesh, device: torch.device, reps: int = 5) -> float:
    """Bandwidth of the band copies' transport, measured with the band copy itself (the kernel,
    or the copy engines under ``OPENDDE_B200_FOLDCP_COPY=dma``): every rank at once copies one
    whole slot of the next rank's window into local memory (4 KB rows) ``reps`` times; returns
    this rank's GB/s of peer reads.
    Collective over the mesh's CP group (its windows must exist: run one op first)."""
    w = _WINDOWS.get(_window_key(mesh))
    if w is None or w.numel < 2:
        raise RuntimeError("peer_copy_gbs needs the mesh's peer windows: run one Fold-CP op first")
    src = w.bases[(w.cp_rank + 1) % w.numel]
    row = 4096
    rows = w.slot_bytes // row
    dst = torch.empty(rows * row, dtype=torch.uint8, device=device)
    plan = [(src, dst.data_ptr(), 1, rows, row, row, row, 0, 0)]
    dma = copy_engine() == "dma"
    kernels.copy_regions(plan, dma=dma)             # warm
    torch.cuda.synchronize(device)
    dist.barrier(group=w.group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        kernels.copy_regions(plan, dma=dma)
    e1.record()
    torch.cuda.synchronize(device)
    dist.barrier(group=w.group)
    return rows * row * reps / (e0.elapsed_time(e1) / 1e3) / 1e9


def release_windows() -> None:
    """Free every cached window (collective over each window's group)."""
    for w in list(_WINDOWS.values()):
        w.release()
    _WINDOWS.clear()


class PeerExchange(DistExchange):
    """DistExchange whose band requests are served from the peers' windows; all-gathers
    (bias planes, single rows) stay NCCL collectives."""

    def __init__(self, mesh, windows_fn=windows_for) -> None:
        super().__init__(mesh)
        self._windows_fn = windows_fn

    def _copy(self, plan: List[CopyRegion]) -> None:
        """Execute a copy plan on the current stream: by the band-copy kernel (one launch per 32
        boxes), or by the copy engines when ``OPENDDE_B200_FOLDCP_COPY=dma``."""
        kernels.copy_regions(plan, dma=copy_engine() == "dma")
        is_remote = getattr(getattr(self, "_w", None), "is_remote", None)
        for r in plan:
            n = r[2] * r[3] * r[4]
            COPY_BYTES["remote" if (is_remote is not None and is_remote(r[0])) else "local"] += n

    def bands(self, local: torch.Tensor, spec: FoldCPPairShardSpec, needs: Sequence[Need]) -> List[torch.Tensor]:
        """Every rectangle ``need(coord)`` of ``needs``, from one snapshot of ``local``."""
        return self._publish_and_gather(local, spec, needs, None)[0]

    def attention_bands(self, local: torch.Tensor, spec: FoldCPPairShardSpec, need: Need,
                        bias_tile: torch.Tensor, transposed: bool, bias_rows: Range):
        """The z band ``need(coord)`` and rows ``bias_rows`` of the triangle-bias plane (all Np
        columns, row pitch rounded to 8 elements), from one snapshot, one barrier and one copy
        launch. ``bias_tile`` [H, x, y] is this rank's tile of the plane in its orientation
        (``transposed``: the ending node's plane, (a, b) = bias of z(b, a)). Only the requested
        bias rows travel, not the whole plane."""
        bands, bias = self._publish_and_gather(local, spec, [need], (bias_tile, transposed, bias_rows))
        return bands[0], bias

    def attention_chunks(self, local: torch.Tensor, spec: FoldCPPairShardSpec, needs: Sequence[Need],
                         bias_tile: torch.Tensor, transposed: bool, bias_rows: Range,
                         consume: Callable[[int, torch.Tensor, torch.Tensor], None]) -> None:
        """attention_bands for a band requested as consecutive chunks ``needs``, overlapped:
        after the snapshot and the barrier, a side stream assembles chunk after chunk (the bias
        rows with the first) while ``consume(i, band_i, bias)`` enqueues chunk i's compute on
        the current stream behind chunk i's copy. Every chunk buffer is allocated before the side
        stream forks, so no memory the current stream still uses is handed to it."""
        plans, outs, bias = self._publish_and_plan(local, spec, needs, (bias_tile, transposed, bias_rows))
        if local.is_cuda and any(plans):
            self._overlap(local.device, plans, lambda i: consume(i, outs[i], bias))
            return
        for i, (plan, out) in enumerate(zip(plans, outs)):
            if plan:
                self._copy(plan)
            consume(i, out, bias)

    def _overlap(self, device, plans, consume_i) -> None:
        """Copy plan after plan on a side stream while ``consume_i(i)`` enqueues chunk i's compute
        on the current stream behind copy i. With an SM reserve (``reserve_sms``, SM copies only),
        the copies after the first and the compute of every chunk but the last run with that many
        SMs left out of the persistent grids, so that copy i + 1 runs beside compute i."""
        r = reserve_sms() if copy_engine() == "sm" else 0
        main = torch.cuda.current_stream(device)
        side = self._side_stream(device)
        side.wait_stream(main)
        done = []
        with torch.cuda.stream(side):
            for i, plan in enumerate(plans):
                if plan:
                    with sm_reserve(r if i > 0 else 0):
                        self._copy(plan)
                ev = torch.cuda.Event()
                ev.record(side)
                done.append(ev)
        for i in range(len(plans)):
            main.wait_event(done[i])
            with sm_reserve(r if i < len(plans) - 1 else 0):
                consume_i(i)

    def _side_stream(self, device) -> "torch.cuda.Stream":
        st = getattr(self, "_side", None)
        if st is None or st.device != device:
            st = torch.cuda.Stream(device=device)
            self._side = st
        return st

    def _publish_and_gather(self, local, spec, needs, bias_req):
        plans, outs, bias = self._publish_and_plan(local, spec, needs, bias_req)
        self._copy([r for plan in plans for r in plan])
        return outs, bias

    def _publish_and_plan(self, local, spec, needs, bias_req):
        """Snapshot (and bias tile) into this rank's slot, barrier, then one copy plan per
        requested band (the bias rows ride with the first) and the band buffers. A band inside
        this rank's own tile is a view of the tile (empty plan)."""
        if not local.is_contiguous():
            raise ValueError("peer exchange publishes contiguous tiles")
        pos_bytes = local.element_size() * (local[0, 0].numel() if local.dim() > 2 else 1)
        tile_bytes = _slot_bytes(local.numel() * local.element_size())
        need_bytes = self._slot_need(local, spec)
        if bias_req is not None:
            bias_tile = bias_req[0]
            eb = bias_tile.element_size()
            ld_t, bias_bytes = _projection_side_bytes(spec, bias_tile.shape[0], eb)
            need_bytes = max(need_bytes, tile_bytes + bias_bytes)
        w = self._windows_fn(self.mesh, need_bytes, local.device)
        self._w = w
        slot = w.slot
        w.slot ^= 1
        ptrs = w.slot_ptrs(slot)
        me = self.mesh.cp_rank
        mine = tile_region(spec, self.coord)
        row_bytes = local.shape[1] * pos_bytes
        publish = [(local.data_ptr(), ptrs[me], 1, local.shape[0], row_bytes, row_bytes, row_bytes, 0, 0)]
        if bias_req is not None:
            H, nx, ny = bias_tile.shape
            if bias_tile.stride(2) != 1:
                raise ValueError("bias tile columns must be contiguous")
            publish.append((bias_tile.data_ptr(), ptrs[me] + tile_bytes, H, nx, ny * eb, bias_tile.stride(1) * eb,
                            ld_t * eb, bias_tile.stride(0) * eb, nx * ld_t * eb))
        self._copy(publish)
        w.barrier()
        outs, plans = [], []
        (mr0, mr1), (mc0, mc1) = mine
        for need in needs:
            (r0, r1), (c0, c1) = need(self.coord)
            if mr0 <= r0 and r1 <= mr1 and mc0 <= c0 and c1 <= mc1:   # inside the own tile: a view
                outs.append(local[r0 - mr0:r1 - mr0, c0 - mc0:c1 - mc0])
                plans.append([])
                continue
            out = local.new_empty((r1 - r0, c1 - c0) + tuple(local.shape[2:]))
            plans.append(band_copy_plan(spec, self.layout, ((r0, r1), (c0, c1)), ptrs, out.data_ptr(), pos_bytes))
            outs.append(out)
        bias = None
        if bias_req is not None:
            _, transposed, rows = bias_req
            ld_b = _round8(spec.n_padded)
            bias = bias_tile.new_empty((bias_tile.shape[0], rows[1] - rows[0], ld_b))
            plans[0] = plans[0] + projection_copy_plan(spec, self.layout, rows, transposed, ptrs, tile_bytes,
                                                       bias_tile.shape[0], eb, ld_t, bias.data_ptr(), ld_b)
        return plans, outs, bias

    def region(self, local: torch.Tensor, spec: FoldCPPairShardSpec, need: Need) -> torch.Tensor:
        return self.bands(local, spec, [need])[0]

    @staticmethod
    def _slot_need(local: torch.Tensor, spec: FoldCPPairShardSpec, c_h: int = 0) -> int:
        """One slot holds a tile snapshot or the a and b projections of a tile (with c_h, by
        default the tile's channel count, channels), whichever is larger, so the windows are
        sized once."""
        elem = local.element_size()
        planes = max(c_h, local.shape[2] if local.dim() > 2 else 1)
        _, side = _projection_side_bytes(spec, planes, elem)
        return max(local.numel() * elem, 2 * side)

    def trimul_chunks(self, local: torch.Tensor, spec: FoldCPPairShardSpec, transposed: bool, c_h: int,
                      project: Callable[[int, int, int], None], parts: Sequence[Range], rows_b: Range,
                      consume: Callable[[int, torch.Tensor, torch.Tensor, int], None]) -> None:
        """trimul_bands with the a band requested as consecutive row chunks ``parts``, overlapped:
        after the projections and the barrier, a side stream copies the b band and then chunk
        after chunk of a, while ``consume(i, a_i, b, Np)`` enqueues chunk i's contraction and
        epilogue on the current stream behind chunk i's copy. All buffers are allocated before
        the side stream forks."""
        elem = local.element_size()
        ld_t, side = _projection_side_bytes(spec, c_h, elem)
        w = self._windows_fn(self.mesh, self._slot_need(local, spec, c_h), local.device)
        self._w = w
        slot = w.slot
        w.slot ^= 1
        ptrs = w.slot_ptrs(slot)
        me = self.mesh.cp_rank
        project(ptrs[me], ptrs[me] + side, ld_t)
        w.barrier()
        n_pad = spec.n_padded
        ld_b = _round8(n_pad)
        b = local.new_empty((c_h, rows_b[1] - rows_b[0], ld_b))
        outs = [local.new_empty((c_h, hi - lo, ld_b)) for lo, hi in parts]
        plans = [projection_copy_plan(spec, self.layout, rows_b, transposed, ptrs, side, c_h, elem, ld_t,
                                      b.data_ptr(), ld_b)]
        plans[0] += projection_copy_plan(spec, self.layout, parts[0], transposed, ptrs, 0, c_h, elem, ld_t,
                                         outs[0].data_ptr(), ld_b)
        for (lo, hi), out in zip(parts[1:], outs[1:]):
            plans.append(projection_copy_plan(spec, self.layout, (lo, hi), transposed, ptrs, 0, c_h, elem, ld_t,
                                              out.data_ptr(), ld_b))
        if local.is_cuda:
            self._overlap(local.device, plans, lambda i: consume(i, outs[i], b, n_pad))
            return
        for i, (plan, out) in enumerate(zip(plans, outs)):
            if plan:
                self._copy(plan)
            consume(i, out, b, n_pad)

    def trimul_bands(self, local: torch.Tensor, spec: FoldCPPairShardSpec, transposed: bool, c_h: int,
                     project: Callable[[int, int, int], None], rows_a: Range, rows_b: Range):
        """The triangle-update operand bands from the peers' projections.

        ``project(a_ptr, b_ptr, ld)`` writes this rank's a and b projections (channel-major
        [c_h][x][ld] over its tile in the projection orientation) into its window; after the
        barrier, a rows ``rows_a`` and b rows ``rows_b`` over all Np columns are assembled from
        every rank's window. Returns (a_band [c_h, |rows_a|, ld_b], b_band, Np). The projections
        cross NVLink instead of z, so no rank recomputes another rank's projections.
        """
        elem = local.element_size()
        ld_t, side = _projection_side_bytes(spec, c_h, elem)
        w = self._windows_fn(self.mesh, self._slot_need(local, spec, c_h), local.device)
        self._w = w
        slot = w.slot
        w.slot ^= 1
        ptrs = w.slot_ptrs(slot)
        me = self.mesh.cp_rank
        project(ptrs[me], ptrs[me] + side, ld_t)
        w.barrier()
        n_pad = spec.n_padded
        ld_b = _round8(n_pad)
        a = local.new_empty((c_h, rows_a[1] - rows_a[0], ld_b))
        b = local.new_empty((c_h, rows_b[1] - rows_b[0], ld_b))
        plan = projection_copy_plan(spec, self.layout, rows_a, transposed, ptrs, 0, c_h, elem, ld_t,
                                    a.data_ptr(), ld_b)
        plan += projection_copy_plan(spec, self.layout, rows_b, transposed, ptrs, side, c_h, elem, ld_t,
                                     b.data_ptr(), ld_b)
        self._copy(plan)
        return a, b, n_pad
