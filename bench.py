"""Benchmark: ms per Pairformer block at N_token=1536 (48-block trunk), bf16, B200.

A step is one forward of the 48-block Pairformer trunk (PairformerStack, c_z=128, c_s=384,
4x32 triangle heads, c_hidden=128, transition x4, 16 single heads) over one synthetic
input (z, s ~ N(0,1), all-ones mask, seed-0 random weights: the reference's default init
zeroes every output projection). ``value`` = device time per step / 48 with inputs resident
in HBM; ``e2e`` = the same through the public API with the step's inputs copied from
pinned host memory and the outputs copied back inside the timed region. The pair tensor
(604 MB) is larger than L2, so no separate flush is needed.

--impl reference times the reference algorithm's CPU path (the oracle restatement of the
reference PyTorch modules; the reference itself is not installed on the GPU box) on the
host cores for a bounded row sample of the same workload, extrapolated to ms per block.

N > 1 GPUs: Fold-CP 2D pair sharding (1x2, 2x2, 2x4 grids) of the same trunk; total work
fixed ("strong" scaling); time = max over ranks. Each step is captured once as a CUDA graph
(kernels, peer copies, NCCL collectives) and replayed; per-kernel times then come from one
extra eager step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

N_TOKEN = 1536
C_Z, C_S, HEADS_PAIR, HEAD_DIM, C_H, N_SINGLE_HEADS = 128, 384, 4, 32, 128, 16
METRIC = "ms per Pairformer block at N_token=1536, 1/2/4/8 B200; tri-attn/tri-mul % peak"
GRIDS = {1: (1, 1), 2: (1, 2), 4: (2, 2), 8: (2, 4)}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ CPU sample
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_block_sample_ms(n: int, rows: int, threads: int, z_full=None) -> float:
    """The reference algorithm on the host (oracle restatement, fp32 torch CPU), one block.

    Every op of the block is row-separable once its O(N^2) shared operands exist: rows
    [0, rows) of each op's output are computed with everything they need (the projections of
    those rows, the full-K contraction and full-key attention for them) and timed x n / rows;
    the triangle update's second operand (b over all N^2 positions, which every output row
    contracts with) is projected once, in full, and timed unscaled.
    """
    from oracle import pairformer_oracle as O
    from opendde_b200.utils import seeded_params
    from opendde_b200.model import PairformerBlock

    torch.set_num_threads(threads)
    blk = PairformerBlock(n_heads=N_SINGLE_HEADS, c_z=C_Z, c_s=C_S)
    p = seeded_params([(k, tuple(v.shape)) for k, v in blk.named_parameters()], seed=0)
    sub = lambda pre: {k[len(pre) + 1:]: v for k, v in p.items() if k.startswith(pre + ".")}  # noqa: E731
    g = torch.Generator().manual_seed(1)
    if z_full is None:
        z_full = torch.randn((n, n, C_Z), generator=g)
    zr = z_full[:rows]
    bias = torch.empty((HEADS_PAIR, n, n)).uniform_(-1, 1, generator=g)
    s = torch.randn((n, C_S), generator=g)
    mask = torch.ones((rows, n))
    scale = n / rows
    t = 0.0
    with torch.no_grad():
        for pre in ("tri_mul_out", "tri_mul_in"):
            q = sub(pre)
            # b over every position (each output row contracts with all of it): once, unscaled
            t0 = time.perf_counter()
            zf = O.layer_norm(z_full, q["layer_norm_in.weight"], q["layer_norm_in.bias"])
            bfull = (torch.sigmoid(O.linear(zf, q["linear_b_g.weight"])) *
                     O.linear(zf, q["linear_b_p.weight"])).permute(2, 0, 1)       # [c_h, j, k]
            t += time.perf_counter() - t0
            del zf
            t0 = time.perf_counter()
            zn = O.layer_norm(zr, q["layer_norm_in.weight"], q["layer_norm_in.bias"])
            a = mask[..., None] * torch.sigmoid(O.linear(zn, q["linear_a_g.weight"])) * O.linear(zn, q["linear_a_p.weight"])
            x = torch.matmul(a.permute(2, 0, 1), bfull.transpose(-1, -2)).permute(1, 2, 0)
            x = O.layer_norm(x, q["layer_norm_out.weight"], q["layer_norm_out.bias"])
            x = O.linear(x, q["linear_z.weight"]) * torch.sigmoid(O.linear(zn, q["linear_g.weight"]))
            t += (time.perf_counter() - t0) * scale
            del a, x, bfull
        for pre in ("tri_att_start", "tri_att_end"):
            q = sub(pre)
            t0 = time.perf_counter()
            x = O.layer_norm(zr, q["layer_norm.weight"], q["layer_norm.bias"])
            _ = O.linear(x, q["linear.weight"])  # the bias rows these output rows contribute
            d = HEAD_DIM
            qq = O.linear(x, q["mha.linear_q.weight"]).view(rows, n, HEADS_PAIR, d).transpose(1, 2) / math.sqrt(d)
            kk = O.linear(x, q["mha.linear_k.weight"]).view(rows, n, HEADS_PAIR, d).transpose(1, 2)
            vv = O.linear(x, q["mha.linear_v.weight"]).view(rows, n, HEADS_PAIR, d).transpose(1, 2)
            for r0 in range(0, rows, 8):
                lg = torch.matmul(qq[r0:r0 + 8], kk[r0:r0 + 8].transpose(-1, -2))
                lg = lg + (1e9 * (mask[r0:r0 + 8] - 1))[:, None, None, :] + bias[None]
                o = torch.matmul(torch.softmax(lg, -1), vv[r0:r0 + 8]).transpose(1, 2)
                gg = torch.sigmoid(O.linear(x[r0:r0 + 8], q["mha.linear_g.weight"])).view(o.shape)
                O.linear((o * gg).reshape(o.shape[0], n, -1), q["mha.linear_o.weight"])
            t += (time.perf_counter() - t0) * scale
        t0 = time.perf_counter()
        O.transition(zr, sub("pair_transition"))
        t += (time.perf_counter() - t0) * scale
        t0 = time.perf_counter()
        apb = sub("attention_pair_bias")
        O.pair_bias(zr, apb)  # pair-bias rows for these output rows (scaled)
        t += (time.perf_counter() - t0) * scale
        t0 = time.perf_counter()
        a = O.layer_norm(s, apb["layernorm_a.weight"], apb["layernorm_a.bias"])
        dd = C_S // N_SINGLE_HEADS
        qs = (O.linear(a, apb["attention.linear_q.weight"], apb["attention.linear_q.bias"]).view(n, N_SINGLE_HEADS, dd).transpose(0, 1) / math.sqrt(dd))
        ks = O.linear(a, apb["attention.linear_k.weight"]).view(n, N_SINGLE_HEADS, dd).transpose(0, 1)
        vs = O.linear(a, apb["attention.linear_v.weight"]).view(n, N_SINGLE_HEADS, dd).transpose(0, 1)
        pb = torch.empty((N_SINGLE_HEADS, n, n)).uniform_(-1, 1, generator=g)
        o = torch.matmul(torch.softmax(torch.matmul(qs, ks.transpose(-1, -2)) + pb, -1), vs)
        O.transition(s, sub("single_transition"))
        t += time.perf_counter() - t0
    return t * 1e3


def cpu_sample_check(threads: int, n: int = 384, rows: int = 32) -> dict:
    """The row-sample extrapolation against one full block of the same algorithm at a size
    where the full block takes seconds: ratio = sampled estimate / full time."""
    from oracle import pairformer_oracle as O
    from opendde_b200.utils import seeded_params
    from opendde_b200.model import PairformerBlock

    torch.set_num_threads(threads)
    blk = PairformerBlock(n_heads=N_SINGLE_HEADS, c_z=C_Z, c_s=C_S)
    p = seeded_params([(k, tuple(v.shape)) for k, v in blk.named_parameters()], seed=0)
    g = torch.Generator().manual_seed(1)
    z = torch.randn((n, n, C_Z), generator=g)
    s = torch.randn((n, C_S), generator=g)
    mask = torch.ones((n, n))
    with torch.no_grad():
        cpu_block_sample_ms(n, rows, threads, z)     # warm-up
        est = cpu_block_sample_ms(n, rows, threads, z)
        t0 = time.perf_counter()
        O.pairformer_block(s, z, mask, p)
        full = (time.perf_counter() - t0) * 1e3
    return {"n": n, "rows": rows, "full_block_ms": full, "sample_estimate_ms": est, "ratio": est / full}


# ------------------------------------------------------------------------------ roofline
# The library states every launch's algorithmic work from its arguments (flops of the
# contraction over the rows / queries / keys that launch processes, or the minimum HBM bytes it
# moves), so on a Fold-CP rank the figures are that rank's share. k_copy_regions is measured
# against the peer-copy bandwidth: its bytes read from peers' windows (over NVLink) per second.
def kernel_entry(name, launches, total_ms, work, unit, peaks, nvlink=None):
    if total_ms <= 0:
        return None
    avg_s = total_ms / launches / 1e3
    base = {"kernel": name, "avg_launch_ms": avg_s * 1e3, "launches": launches}
    if name in ("k_copy_regions", "dma_copy_regions") and nvlink is not None and nvlink.get("remote_bytes"):
        rb = nvlink["remote_bytes"] / launches
        ach = rb / avg_s / 1e9
        peak = nvlink["peak_gbs"]
        base.update({"bound": "nvlink", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                     "traffic": None, "work_per_launch": rb, "work_unit": "byte read from peers",
                     "peak_kind": nvlink["peak_kind"]})
        return base
    if not work or not unit:
        return None
    per = work / launches
    if unit == "flop":
        ach = per / avg_s / 1e12
        peak = peaks["bf16_tflops_sustained"]
        base.update({"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                     "traffic": read_traffic(name, per), "work_per_launch": per, "work_unit": "flop",
                     "peak_kind": f"bf16 dense sustained ({peaks['source']})"})
    else:
        ach = per / avg_s / 1e9
        peak = peaks["hbm_gbs"]
        base.update({"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                     "traffic": read_traffic(name, per), "work_per_launch": per, "work_unit": "byte",
                     "peak_kind": f"HBM copy ({peaks['source']})"})
    return base


def read_traffic(kernel: str, work_per_launch: float):
    """DRAM bytes per launch for `kernel` from the committed ncu summary, when this launch
    does the same work as the captured one (the summary's third column), else None."""
    p = os.path.join(ROOT, "profiles", "dram_traffic_per_launch.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel:
                try:
                    traffic, ref_work = float(parts[1]), float(parts[2])
                except ValueError:
                    return None
                return traffic if abs(work_per_launch - ref_work) <= 1e-3 * ref_work else None
    return None


def current_mesh():
    from opendde_b200.distributed.foldcp import runtime
    return runtime.current_mesh()


def parity_vs_one_gpu(stack, s_dev, z_dev, m_dev, blocks, rank, barrier):
    """The first ``blocks`` blocks of the timed trunk, run under Fold-CP on every rank and then
    on rank 0 alone (single-device mode): rel-L2 of the final z and s between the two."""
    from opendde_b200.model import PairformerStack
    sub = PairformerStack(n_blocks=0, n_heads=N_SINGLE_HEADS, c_z=C_Z, c_s=C_S)
    sub.blocks = torch.nn.ModuleList(list(stack.blocks)[:blocks])
    out = None
    with torch.no_grad():
        s_d, z_d = sub(s_dev, z_dev, m_dev)
        barrier()
        if rank == 0:
            old = os.environ.get("OPENDDE_FOLDCP_MODE")
            os.environ["OPENDDE_FOLDCP_MODE"] = "single"
            try:
                s_1, z_1 = sub(s_dev, z_dev, m_dev)
            finally:
                os.environ["OPENDDE_FOLDCP_MODE"] = old
            rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()  # noqa: E731
            out = {"blocks": blocks, "rel_l2_z": rel(z_d, z_1), "rel_l2_s": rel(s_d, s_1),
                   "against": "the same seeded trunk on 1 GPU (bf16)"}
        barrier()
    return out


# ------------------------------------------------------------------------------ C1 / C2
def executed_key_fraction(mask: torch.Tensor, tile: int = 128) -> float:
    """Fraction of the (row, key) pairs whose 128-key tile the attention core executes. The core
    skips a key tile of a row when every key in it is masked while the row has a key of mask 1
    (exp() of those logits is exactly 0 in the reference too); a row with no such key attends
    uniformly over all keys, so none of its tiles is skipped."""
    n_rows, n = mask.shape
    n_tiles = (n + tile - 1) // tile
    full = mask >= 1.0
    row_full = full.any(dim=1, keepdim=True)
    live = full | ~row_full
    pad = n_tiles * tile - n
    live_t = torch.nn.functional.pad(live, (0, pad), value=False).view(n_rows, n_tiles, tile)
    run = live_t.any(dim=2)                                         # tile executed
    keys = torch.full((n_tiles,), tile, device=mask.device)
    keys[-1] = n - (n_tiles - 1) * tile
    return float((run.float() * keys).sum() / (n_rows * n))


def run_op_workload(args, kind):
    """Standalone triangle attention (C1: start and end, N = 384 / 768 / 1536, last 10 % of tokens
    padded) or triangle multiplicative update (C2: outgoing and incoming, N = 1024), bf16, one
    GPU: ms per call through the module forward (inputs resident), and the core kernel's
    fraction of the measured peak from the library's per-launch work and CUDA-event times."""
    from opendde_b200 import _abi
    from opendde_b200.model import (TriangleAttention, TriangleMultiplicationIncoming,
                                    TriangleMultiplicationOutgoing)
    from opendde_b200.utils import make_inputs, seeded_init_

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    if kind == "c1":
        sizes, pad, core = [384, 768, 1536], 0.1, "k_triatt_core"
        mods = [("start", TriangleAttention(c_in=C_Z, c_hidden=HEAD_DIM, no_heads=HEADS_PAIR, starting=True)),
                ("end", TriangleAttention(c_in=C_Z, c_hidden=HEAD_DIM, no_heads=HEADS_PAIR, starting=False))]
        metric = "ms per standalone triangle-attention call (C1), bf16; tri-attn % peak"
    else:
        sizes, pad, core = [1024], 0.0, "k_trimul_bgemm"
        mods = [("out", TriangleMultiplicationOutgoing(c_z=C_Z, c_hidden=C_H)),
                ("in", TriangleMultiplicationIncoming(c_z=C_Z, c_hidden=C_H))]
        metric = "ms per standalone triangle multiplicative update call (C2), bf16; tri-mul % peak"
    for _, m in mods:
        seeded_init_(m, seed=0)
        m.to(dev)
    rows = []
    st = torch.cuda.current_stream()
    with ClockSampler(0) as clk:
        for n in sizes:
            _, z, mask = make_inputs(n, c_z=C_Z, seed=1, pad_frac=pad, with_s=False)
            zb, md = z.to(dev, torch.bfloat16), mask.to(dev)
            for name, m in mods:
                with torch.no_grad():
                    for _ in range(args.warmup):
                        m(zb, mask=md)
                    torch.cuda.synchronize()
                    _abi.profile_enable(True)
                    _abi.profile_report()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    for _ in range(args.steps):
                        m(zb, mask=md)
                    e1.record(st)
                    torch.cuda.synchronize()
                    _abi.profile_enable(False)
                    prof = _abi.profile_report()
                ms = e0.elapsed_time(e1) / args.steps
                e = kernel_entry(core, *prof[core], peaks) if core in prof else None
                if e is not None and kind == "c1":
                    # the stated flops count every key (as the reference computes them); the
                    # core skips fully masked key tiles, so also report the executed work
                    frac_run = executed_key_fraction(md if name == "start" else md.t())
                    e.update({"executed_key_fraction": frac_run,
                              "executed_work_per_launch": e["work_per_launch"] * frac_run,
                              "achieved_executed": e["achieved"] * frac_run,
                              "frac_executed": e["frac"] * frac_run})
                kern = {k: round(v[1] / v[0], 4) for k, v in prof.items()}
                rows.append({"n": n, "op": name, "ms_per_call": ms, "core": e, "kernels_ms_per_launch": kern})
    assert _abi.device_status() == 0, "a device-side bounded wait timed out"
    big = [r for r in rows if r["n"] == sizes[-1]]
    value = statistics.mean(r["ms_per_call"] for r in big)
    print(json.dumps({
        "metric": metric, "value": value, "unit": "ms/call", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic: z ~ N(0,1), last {int(pad * 100)} % of tokens padded, seed-0 N(0,1/fan_in) weights",
        "config": {"workload": f"{kind}_" + "_".join(str(n) for n in sizes), "c_z": C_Z,
                   "l2": "inputs at N >= 768 larger than L2; smaller ones repeat from L2"},
        "roofline": big[0]["core"], "sweep": rows, "clocks": clk.summary(),
    }), flush=True)


# ------------------------------------------------------------------------------ heads
def run_heads_workload(args):
    """The pair work downstream of the stack at N = --n-token on the trunk's pair width, bf16, one
    GPU: the distogram logits + contact probabilities (96 bins), the confidence head's pair input
    and its pae / pde logits (64 bins each, fp32 out), and the diffusion pair conditioning
    (c_z -> 128). ms per call through the module API (inputs resident) and every kernel's fraction
    of the measured HBM (or bf16) peak from the library's per-launch work and CUDA-event times."""
    from opendde_b200 import _abi
    from opendde_b200.model import ConfidencePairHead, DiffusionPairConditioning, DistogramHead
    from opendde_b200.model.trunk_init import LazyRelativePositionEncodingFeatures
    from opendde_b200.utils import seeded_init_

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    n, c_s_in = args.n, 449
    g = torch.Generator().manual_seed(1)
    z = torch.randn((n, n, C_Z), generator=g).to(dev, torch.bfloat16)
    s_in = torch.randn((n, c_s_in), generator=g).to(dev, torch.bfloat16)
    coords = (torch.randn((n, 3), generator=g) * 20.0).to(dev)
    chains = torch.arange(n) * 4 // n
    ids = [t.to(dev) for t in (chains, torch.arange(n) - chains * 300, chains % 2, torch.arange(n), chains // 2)]
    relp = LazyRelativePositionEncodingFeatures(*ids, r_max=32, s_max=2)
    dh, ch = DistogramHead(C_Z, 96), ConfidencePairHead(c_z=C_Z, c_s_inputs=c_s_in)
    dc = DiffusionPairConditioning(C_Z, 128)
    for i, m in enumerate((dh, ch, dc)):
        seeded_init_(m, seed=i)
        m.to(dev)
    zp = torch.empty_like(z)
    ops = [("distogram", lambda: dh.contact_probs(z, 2.25, 25.75, 96, 8.0)),
           ("confidence_pair_input", lambda: ch.embed_pair_tile(s_in, coords, z, zp)),
           ("confidence_pae_pde", lambda: ch.pair_logits(zp)),
           ("diffusion_pair_cond", lambda: dc.prepare_cache(relp, z))]
    rows = []
    st = torch.cuda.current_stream()
    with ClockSampler(0) as clk:
        for name, fn in ops:
            with torch.no_grad():
                for _ in range(args.warmup):
                    fn()
                torch.cuda.synchronize()
                _abi.profile_enable(True)
                _abi.profile_report()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(args.steps):
                    fn()
                e1.record(st)
                torch.cuda.synchronize()
                _abi.profile_enable(False)
                prof = _abi.profile_report()
            ents = {}
            for k, (launches, total, work, unit) in prof.items():
                e = kernel_entry(k, launches, total, work, unit, peaks)
                ents[k] = {"ms_per_call": total / args.steps, "launches_per_call": launches / args.steps,
                           "bound": e and e["bound"], "achieved": e and e["achieved"], "frac": e and e["frac"],
                           "unit": e and e["unit"]}
            rows.append({"op": name, "ms_per_call": e0.elapsed_time(e1) / args.steps, "kernels": ents})
    assert _abi.device_status() == 0, "a device-side bounded wait timed out"
    value = sum(r["ms_per_call"] for r in rows)
    dom = max(((k, v) for r in rows for k, v in r["kernels"].items()), key=lambda kv: kv[1]["ms_per_call"])
    print(json.dumps({
        "metric": "ms for the pair heads and the diffusion pair conditioning after the trunk, bf16",
        "value": value, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": value, "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: z ~ N(0,1), s_inputs ~ N(0,1), coordinates ~ N(0, 20 A), four chains; seeded weights",
        "config": {"workload": f"pair_heads_N{n}", "n_token": n, "c_z": C_Z, "distogram_bins": 96,
                   "pae_pde_bins": 64, "c_z_pair_diffusion": 128,
                   "l2": "inputs larger than L2 (pair tensor %d MB)" % (n * n * C_Z * 2 // 10**6)},
        "dominant_kernel": {"kernel": dom[0], **dom[1]}, "ops": rows, "clocks": clk.summary(),
    }), flush=True)


# ------------------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["trunk", "c1", "c2", "heads"], default="trunk",
                    help="trunk: the 48-block trunk (the headline); c1 / c2: standalone triangle attention / "
                         "triangle multiplicative update at their configurations (1 GPU); heads: the pair "
                         "heads and the diffusion pair conditioning after the trunk (1 GPU)")
    # "--n-token" first: torchrun resolves abbreviated options even after the script name, and a
    # bare "--n" is ambiguous to it
    ap.add_argument("--n-token", "--n", dest="n", type=int, default=N_TOKEN)
    ap.add_argument("--pad-frac", type=float, default=0.0,
                    help="fraction of trailing tokens masked as padding (config C4: 0.07)")
    ap.add_argument("--blocks", type=int, default=48)
    ap.add_argument("--cpu-rows", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--parity-blocks", type=int, default=2,
                    help="N > 1: blocks of the same trunk run once more under Fold-CP and on rank 0 alone; "
                         "the line's parity field is their rel-L2")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="replay each step as one CUDA graph (auto: on for N > 1, where the per-op host "
                         "work and collective launches would otherwise show between short kernels)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    cores = os.cpu_count() or 1
    if args.workload != "trunk" and args.impl == "ours":
        if rank == 0:
            if args.workload == "heads":
                run_heads_workload(args)
            else:
                run_op_workload(args, args.workload)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        rows = max(8, min(args.cpu_rows, args.n))
        for _ in range(args.warmup):
            cpu_block_sample_ms(args.n, rows, cores)
        vals = [cpu_block_sample_ms(args.n, rows, cores) for _ in range(args.steps)]
        v = statistics.median(vals)
        sample = (f"rows 0..{rows - 1} of every op of one block at N={args.n} (row-separable; the rows' "
                  f"projections, full-K contractions and full-key attention), scaled x{args.n}/{rows}; "
                  f"fp32 torch CPU restatement of the reference modules")
        print(json.dumps({
            "metric": METRIC, "value": v, "unit": "ms/block", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": v * args.blocks,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"pairformer_trunk_{args.blocks}blk_N{args.n}", "n_token": args.n,
                       "c_z": C_Z, "c_s": C_S, "blocks": args.blocks},
            "cpu_baseline": {"value": v, "unit": "ms/block", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "ms/block", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    from opendde_b200 import _abi
    from opendde_b200.model import PairformerStack
    from opendde_b200.utils import make_inputs, seeded_init_

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    distributed = world > 1
    if distributed:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        os.environ["OPENDDE_FOLDCP_MODE"] = "distributed"
        os.environ["OPENDDE_FOLDCP_SIZE_CP"] = str(world)
        os.environ["OPENDDE_FOLDCP_SIZE_DP"] = "1"
        r_, c_ = GRIDS[world]
        os.environ["OPENDDE_FOLDCP_MESH"] = f"{r_}x{c_}"

    stack = PairformerStack(n_blocks=args.blocks, n_heads=N_SINGLE_HEADS, c_z=C_Z, c_s=C_S)
    seeded_init_(stack, seed=0)
    stack = stack.to(dev)
    s0, z0, m0 = make_inputs(args.n, c_z=C_Z, c_s=C_S, seed=1, pad_frac=args.pad_frac)
    z_dev = z0.to(dev, torch.bfloat16)
    s_dev = s0.to(dev, torch.bfloat16)
    m_dev = m0.to(dev)
    z_host = z0.to(torch.bfloat16).pin_memory()
    s_host = s0.to(torch.bfloat16).pin_memory()
    m_host = m0.pin_memory()
    z_out_host = torch.empty_like(z_host).pin_memory()
    s_out_host = torch.empty_like(s_host).pin_memory()

    def barrier():
        if distributed:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def step_resident():
        with torch.no_grad():
            return stack(s_dev, z_dev, m_dev)

    def step_e2e():
        with torch.no_grad():
            zz = z_host.to(dev, non_blocking=True)
            ss = s_host.to(dev, non_blocking=True)
            mm = m_host.to(dev, non_blocking=True)
            so, zo = stack(ss, zz, mm)
            z_out_host.copy_(zo, non_blocking=True)
            s_out_host.copy_(so, non_blocking=True)

    for _ in range(args.warmup):
        step_resident()
    step_e2e()
    barrier()

    use_graph = args.graph == "on" or (args.graph == "auto" and distributed)
    graphs = {}
    if use_graph:
        # one CUDA graph per step kind (kernels, peer copies and NCCL collectives of all blocks),
        # captured after the eager warm-up has created every window, communicator and workspace
        for name, fn in (("resident", step_resident), ("e2e", step_e2e)):
            graphs[name] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphs[name]):
                fn()
        barrier()
        for name in graphs:   # warm replay
            graphs[name].replay()
        barrier()
    def run_resident():
        graphs["resident"].replay() if use_graph else step_resident()

    def run_e2e():
        graphs["e2e"].replay() if use_graph else step_e2e()

    st = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches_per_step = None
    copy_bytes = {"remote": 0, "local": 0}
    if distributed:
        from opendde_b200.distributed.foldcp import peer as foldcp_peer
    if use_graph:
        # per-kernel launch times from one eager step (graph replays carry no per-launch events)
        _abi.profile_enable(True)
        _abi.profile_report()
        if distributed:
            foldcp_peer.reset_copy_bytes()
        l0 = _abi.launch_count()
        step_resident()
        launches_per_step = _abi.launch_count() - l0
        _abi.profile_enable(False)
        prof = _abi.profile_report()
        if distributed:
            copy_bytes = foldcp_peer.reset_copy_bytes()
        barrier()

    # ---- timed: resident inputs (value); eager runs carry per-kernel events (roofline)
    if not use_graph:
        _abi.profile_enable(True)
        _abi.profile_report()  # clear
        if distributed:
            foldcp_peer.reset_copy_bytes()
    launches0 = _abi.launch_count()
    with ClockSampler(local_rank) as clk:
        barrier()
        ev0.record(st)
        for _ in range(args.steps):
            run_resident()
        ev1.record(st)
        barrier()
    if use_graph:
        launches = launches_per_step * args.steps
    else:
        launches = _abi.launch_count() - launches0
        _abi.profile_enable(False)
        prof = _abi.profile_report()
        if distributed:
            copy_bytes = foldcp_peer.reset_copy_bytes()
    ms_step = ev0.elapsed_time(ev1) / args.steps

    # ---- timed: end to end through the public API with host buffers
    barrier()
    ev0.record(st)
    for _ in range(args.steps):
        run_e2e()
    ev1.record(st)
    barrier()
    ms_e2e = ev0.elapsed_time(ev1) / args.steps
    assert _abi.device_status() == 0, "a device-side bounded wait timed out"

    if distributed:
        t = torch.tensor([ms_step, ms_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_step, ms_e2e = t.tolist()

    # ---- N > 1: the transport's measured bandwidth, and parity against one GPU at reduced depth
    nvlink = None
    parity = None
    if distributed:
        mesh = current_mesh()
        gbs = foldcp_peer.peer_copy_gbs(mesh, dev) if foldcp_peer.transport_choice("nccl") == "peer" else None
        if gbs is not None:
            t = torch.tensor([gbs], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            nvlink = {"peak_gbs": t.item(), "remote_bytes": copy_bytes["remote"],
                      "peak_kind": "peer copy measured in this run with pf_copy_regions (min over ranks)"}
        parity = parity_vs_one_gpu(stack, s_dev, z_dev, m_dev, args.parity_blocks, rank, barrier)

    peaks = load_peaks()
    clocks = clk.summary()
    kernels = {k: {"launches": v[0], "total_ms": v[1], "share": None, "work": v[2], "work_unit": v[3]}
               for k, v in prof.items()}
    tot = sum(v[1] for v in prof.values()) or 1.0
    for k in kernels:
        kernels[k]["share"] = kernels[k]["total_ms"] / tot
    entries = {k: kernel_entry(k, v[0], v[1], v[2], v[3], peaks, nvlink) for k, v in prof.items()}
    for k, e in entries.items():
        if e is not None:
            kernels[k]["roofline_frac"] = e["frac"]
    # the roofline entry is the dominant kernel of the timed region (most device time)
    dom = max(prof.items(), key=lambda kv: kv[1][1])[0] if prof else None
    roofline = entries.get(dom)

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = max(8, min(args.cpu_rows, args.n))
        v = cpu_block_sample_ms(args.n, rows, cores)
        cpu_baseline = {"value": v, "unit": "ms/block", "cores": cores, "kind": "port", "cpu": cpu_model(),
                        "sample": f"rows 0..{rows - 1} of every op of one block at N={args.n}, scaled x{args.n}/{rows} "
                                  "(the triangle update's full b projection timed once, unscaled); fp32 torch CPU "
                                  "restatement of the reference modules",
                        "sample_check": cpu_sample_check(cores)}

    # device memory: the peak held by one rank (max over ranks), the pair tensor's share of it
    mem_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    if distributed:
        t = torch.tensor([mem_gb], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        mem_gb = t.item()
    z_bytes = z_host.numel() * 2
    h2d = z_bytes + s_host.numel() * 2 + m_host.numel() * 4
    d2h = z_bytes + s_host.numel() * 2
    if rank == 0:
        grid = GRIDS.get(world, (1, world))
        out = {
            "metric": METRIC,
            "value": ms_step / args.blocks,
            "unit": "ms/block",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": ("synthetic: z,s ~ N(0,1), " + (f"last {args.pad_frac:.0%} of tokens padded" if args.pad_frac > 0
                                                       else "all-ones mask") + ", seed-0 N(0,1/fan_in) weights"),
            "config": {"workload": f"pairformer_trunk_{args.blocks}blk_N{args.n}_bf16", "n_token": args.n,
                       "c_z": C_Z, "c_s": C_S, "blocks": args.blocks, "grid": f"{grid[0]}x{grid[1]}",
                       "pad_frac": args.pad_frac,
                       "l2": f"inputs larger than L2 (pair tensor {z_bytes / 1e6:.0f} MB)"},
            "memory": {"max_allocated_gb_per_rank": mem_gb, "pair_tensor_gb": z_bytes / 1e9},
            "e2e": {"value": ms_e2e / args.blocks, "unit": "ms/block", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roofline,
            "tri_attn": entries.get("k_triatt_core"),
            "tri_mul": entries.get("k_trimul_bgemm"),
            "parity": parity,
            "kernels": kernels,
            "gpu_launches": launches,
            "cuda_graph": use_graph,
            "clocks": clocks,
            "cpu_baseline": cpu_baseline,
        }
        print(json.dumps(out), flush=True)
    # graphs holding NCCL calls must be destroyed before the process group: drop every reference
    graphs.clear()
    torch.cuda.synchronize()
    if distributed:
        from opendde_b200.distributed.foldcp import clear_mesh_cache
        torch.distributed.barrier()
        clear_mesh_cache()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
