"""Test support for the Fold-CP drivers.

``OracleBandOps``: the local band computations of ``opendde_b200.distributed.foldcp.ops``
restated on the CPU oracle (fp32 torch), with the same semantics, so the exchange and
assembly logic runs on CPU process groups (gloo) and is checked against the serial oracle.

``ThreadMesh``: R x C ranks emulated as threads of one process sharing one device; its
transport copies band intersections straight out of the peers' tiles ("copy"), or, on a GPU,
runs the peer-memory transport with in-process windows ("peer"). It runs the real drivers (and,
on a GPU, the real kernels) for every rank of a mesh on a single device.
"""

from __future__ import annotations

import ctypes
import math
import threading
from typing import Callable, Dict, List, Optional, Tuple

import torch

from types import SimpleNamespace

from oracle import pairformer_oracle as O
from opendde_b200.distributed.foldcp.exchange import copy_intersection, tile_region
from opendde_b200.distributed.foldcp.layout import FoldCP2DLayout
from opendde_b200.distributed.foldcp.peer import PeerExchange


def _params(module) -> Dict[str, torch.Tensor]:
    return {k: v.detach() for k, v in module.named_parameters()}


class OracleBandOps:
    """Same contract as KernelOps, computed by the oracle's primitives (fp32)."""

    def bias_dtype(self, z_dtype):
        return torch.float32

    def trimul(self, module, za, zb, ma, mb, zg, zo):
        p = _params(module)
        ln_w, ln_b = p["layer_norm_in.weight"], p["layer_norm_in.bias"]
        xa = O.layer_norm(za, ln_w, ln_b)
        xb = O.layer_norm(zb, ln_w, ln_b)
        a = ma[..., None] * torch.sigmoid(O.linear(xa, p["linear_a_g.weight"])) * O.linear(xa, p["linear_a_p.weight"])
        b = mb[..., None] * torch.sigmoid(O.linear(xb, p["linear_b_g.weight"])) * O.linear(xb, p["linear_b_p.weight"])
        x = torch.einsum("ikc,jkc->ijc", a, b)
        x = O.layer_norm(x, p["layer_norm_out.weight"], p["layer_norm_out.bias"])
        x = O.linear(x, p["linear_z.weight"])
        g = torch.sigmoid(O.linear(O.layer_norm(zg, ln_w, ln_b), p["linear_g.weight"]))
        zo += x * g

    def trimul_project(self, module, z_view, m_view, a_ptr, b_ptr, ld):
        """a, b of a tile view written channel-major [c_h][rows][ld] (fp32) at raw host
        addresses, like the library's pf_trimul_project."""
        p = _params(module)
        ln_w, ln_b = p["layer_norm_in.weight"], p["layer_norm_in.bias"]
        x = O.layer_norm(z_view, ln_w, ln_b)
        rows, cols = z_view.shape[:2]
        for name, ptr in (("a", a_ptr), ("b", b_ptr)):
            v = m_view[..., None] * torch.sigmoid(O.linear(x, p[f"linear_{name}_g.weight"])) * \
                O.linear(x, p[f"linear_{name}_p.weight"])
            out = torch.zeros((v.shape[2], rows, ld), dtype=torch.float32)
            out[:, :, :cols] = v.permute(2, 0, 1)
            ctypes.memmove(ptr, out.data_ptr(), out.numel() * 4)

    def trimul_combine(self, module, a, b, n_k, zg, zo):
        p = _params(module)
        ln_w, ln_b = p["layer_norm_in.weight"], p["layer_norm_in.bias"]
        x = torch.einsum("cik,cjk->ijc", a[:, :, :n_k], b[:, :, :n_k])
        x = O.layer_norm(x, p["layer_norm_out.weight"], p["layer_norm_out.bias"])
        x = O.linear(x, p["linear_z.weight"])
        g = torch.sigmoid(O.linear(O.layer_norm(zg, ln_w, ln_b), p["linear_g.weight"]))
        zo += x * g

    def triatt_bias(self, module, z_view, out):
        p = _params(module)
        x = O.layer_norm(z_view, p["layer_norm.weight"], p["layer_norm.bias"])
        out.copy_(O.linear(x, p["linear.weight"]).permute(2, 0, 1))

    def triatt(self, module, zs, m, bias, zo, q_col0, n_q, n_valid):
        p = _params(module)
        H, d = module.no_heads, module.c_hidden
        rows = zs.shape[0]
        x = O.layer_norm(zs, p["layer_norm.weight"], p["layer_norm.bias"])
        xq = x[:, q_col0:q_col0 + n_q]
        xk = x[:, :n_valid]
        q = O.linear(xq, p["mha.linear_q.weight"]).view(rows, n_q, H, d).transpose(1, 2) / math.sqrt(d)
        k = O.linear(xk, p["mha.linear_k.weight"]).view(rows, n_valid, H, d).transpose(1, 2)
        v = O.linear(xk, p["mha.linear_v.weight"]).view(rows, n_valid, H, d).transpose(1, 2)
        logits = torch.matmul(q, k.transpose(-1, -2))
        logits = logits + (module.inf * (m[:, :n_valid] - 1.0))[:, None, None, :]
        logits = logits + bias[None, :, :, :n_valid]
        o = torch.matmul(torch.softmax(logits, -1), v).transpose(1, 2)
        g = torch.sigmoid(O.linear(xq, p["mha.linear_g.weight"])).view(rows, n_q, H, d)
        zo += O.linear((o * g).reshape(rows, n_q, H * d), p["mha.linear_o.weight"])

    def transition(self, module, x2d):
        x2d += O.transition(x2d, _params(module))

    def apb_pair_bias(self, module, z_view, out):
        out.copy_(O.pair_bias(z_view, _params(module)))

    def apb_rows(self, module, s, s_rows, bias_rows, q_row0):
        p = _params(module)
        H = module.n_heads
        n, c = s.shape
        nq = s_rows.shape[0]
        d = c // H
        a = O.layer_norm(s, p["layernorm_a.weight"], p["layernorm_a.bias"])
        aq = a[q_row0:q_row0 + nq]
        q = O.linear(aq, p["attention.linear_q.weight"], p["attention.linear_q.bias"]).view(nq, H, d).transpose(0, 1)
        q = q / math.sqrt(d)
        k = O.linear(a, p["attention.linear_k.weight"]).view(n, H, d).transpose(0, 1)
        v = O.linear(a, p["attention.linear_v.weight"]).view(n, H, d).transpose(0, 1)
        o = torch.matmul(torch.softmax(torch.matmul(q, k.transpose(-1, -2)) + bias_rows, -1), v).transpose(0, 1)
        g = torch.sigmoid(O.linear(aq, p["attention.linear_g.weight"])).view(nq, H, d)
        s_rows += O.linear((o * g).reshape(nq, c), p["attention.linear_o.weight"])

    def single_transition(self, module, s_rows):
        s_rows += O.transition(s_rows, _params(module))


class _ThreadExchange:
    """One rank's view of a ThreadMesh transport."""

    def __init__(self, mesh: "ThreadMesh", rank: int) -> None:
        self.m = mesh
        self.rank = rank
        self.layout = mesh.layout
        self.coord = mesh.layout.to_coord(rank)

    def region(self, local, spec, need):
        m = self.m
        m.slots[self.rank] = local
        m.wait()
        want = need(self.coord)
        (r0, r1), (c0, c1) = want
        out = local.new_empty((r1 - r0, c1 - c0) + tuple(local.shape[2:]))
        for q in range(self.layout.numel):
            copy_intersection(out, want, m.slots[q], tile_region(spec, self.layout.to_coord(q)))
        m.wait()
        return out

    def all_gather(self, t, axis):
        m = self.m
        m.slots[self.rank] = t.contiguous()
        m.wait()
        R, C = self.layout.shape
        r, c = self.coord
        if axis == "2d":
            members = range(R * C)
        elif axis == "row":
            members = [self.layout.to_linear((r, cc)) for cc in range(C)]
        else:
            members = [self.layout.to_linear((rr, c)) for rr in range(R)]
        out = torch.stack([m.slots[q].clone() for q in members], 0)
        m.wait()
        return out


class _ThreadWindows:
    """One rank's view of a ThreadMesh's peer windows (device buffers of one process); the
    barrier synchronises the device and then the threads."""

    def __init__(self, mesh: "ThreadMesh") -> None:
        self.m = mesh
        self.slot = 0

    @property
    def slot_bytes(self) -> int:
        return self.m.win_bytes

    def slot_ptrs(self, slot: int) -> List[int]:
        return [b.data_ptr() + slot * self.m.win_bytes for b in self.m.win_bufs]

    def is_remote(self, ptr: int) -> bool:
        mine = self.m.win_views.index(self)
        return any(b.data_ptr() <= ptr < b.data_ptr() + 2 * self.m.win_bytes
                   for q, b in enumerate(self.m.win_bufs) if q != mine)

    def barrier(self) -> None:
        if self.m.win_bufs and self.m.win_bufs[0].is_cuda:
            torch.cuda.synchronize()
        self.m.wait()


class ThreadPeerExchange(PeerExchange):
    """The peer-memory transport (snapshot, barrier, pf_copy_regions gather) on a ThreadMesh:
    the windows are buffers of this process, the all-gathers those of _ThreadExchange."""

    def __init__(self, mesh: "ThreadMesh", rank: int) -> None:
        self._t = _ThreadExchange(mesh, rank)
        self.m = mesh
        fake = SimpleNamespace(layout=mesh.layout, coord=self._t.coord, cp_rank=rank)
        super().__init__(fake, windows_fn=lambda _m, nbytes, dev: mesh.peer_windows(rank, nbytes, dev))

    def all_gather(self, t, axis):
        return self._t.all_gather(t, axis)

    def _copy(self, plan):
        if self.m.win_bufs and self.m.win_bufs[0].is_cuda:
            return super()._copy(plan)
        apply_copy_plan(plan)


def apply_copy_plan(plan) -> None:
    """Host execution of a pf_copy_regions plan on CPU memory (byte boxes)."""
    for src, dst, planes, rows, row_bytes, sp, dp, spp, dpp in plan:
        for c in range(planes):
            for r in range(rows):
                ctypes.memmove(dst + c * dpp + r * dp, src + c * spp + r * sp, row_bytes)


class ThreadMesh:
    """Run ``fn(exchange, rank)`` for every rank of an R x C mesh as threads."""

    def __init__(self, shape: Tuple[int, int], timeout: float = 300.0, transport: str = "copy") -> None:
        self.layout = FoldCP2DLayout(shape)
        self.barrier = threading.Barrier(self.layout.numel, timeout=timeout)
        self.slots: List[Optional[torch.Tensor]] = [None] * self.layout.numel
        self.transport = transport
        self.lock = threading.Lock()
        self.win_bytes = 0
        self.win_bufs: List[torch.Tensor] = []
        self.win_views = [_ThreadWindows(self) for _ in range(self.layout.numel)]

    def wait(self) -> None:
        self.barrier.wait()

    def peer_windows(self, rank: int, nbytes: int, device) -> _ThreadWindows:
        with self.lock:
            need = (nbytes + 255) // 256 * 256
            if self.win_bytes < need:
                if self.win_bufs:
                    raise RuntimeError("thread windows cannot grow once in use")
                self.win_bufs = [torch.empty(2 * need, dtype=torch.uint8, device=device)
                                 for _ in range(self.layout.numel)]
                self.win_bytes = need
        return self.win_views[rank]

    def run(self, fn: Callable) -> list:
        n = self.layout.numel
        results: list = [None] * n
        errors: list = []
        make = ThreadPeerExchange if self.transport == "peer" else _ThreadExchange

        def body(rank):
            try:
                results[rank] = fn(make(self, rank), rank)
            except BaseException as e:  # noqa: BLE001 - re-raised below
                errors.append(e)
                self.barrier.abort()

        threads = [threading.Thread(target=body, args=(r,)) for r in range(n)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        real = [e for e in errors if not isinstance(e, threading.BrokenBarrierError)]
        if real or errors:
            raise (real or errors)[0]
        return results
