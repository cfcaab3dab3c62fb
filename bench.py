#!/usr/bin/env python
"""bench.py -- beacon hot-path benchmark on B200.

Headline workload: bf16 causal attention forward + backward, B=8, H=32, S=4096,
D=128, Q/K/V/dO i.i.d. N(0,1) (synthetic, seeded), scale 1/sqrt(128), fp32
softmax statistics; the B*H = 256 heads are sharded across ranks (strong
scaling, no collective on the data path).  One step = attention_adjoint_fwd +
attention_adjoint_bwd through the C ABI, the drop-in path of the reference's
adjoint entry (the backward is not given O and recomputes it).  TFLOP/s use the
FlashAttention convention: fwd 2*B*H*S^2*D (causal), bwd 2.5x fwd; recompute
work is not counted.

Also reported on the same JSON line:
  "gemm":      4096^3 bf16 GEMM, columns of B sharded across ranks, L2 flushed
               between timed iterations;
  "with_out":  the same fwd+bwd when the backward is given O (no recompute);
  "roofline":  the dominant kernel (k_attn_bwd_dkdv) timed live with CUDA events on
               its launch stream against the measured dense bf16 peak;
  "cpu_baseline": the CPU oracle on a bounded sample of heads (rank 0, N=1);
  "e2e":       the step with pinned-host inputs copied in and results copied out,
               pipelined over head chunks (copies in / compute / copies out overlap);
  "block":     one pre-norm Llama block forward (batch 4 x seq 2048, d_model 4096,
               32 x 128 heads, SwiGLU hidden 14336), one replica per rank;
  "gqa":       long-context grouped-query causal forward (64 query heads, 8 KV heads,
               S=32768, D=128), KV groups sharded across ranks;
  "block_backward": the backward operators at the block's shapes (SwiGLU MLP, the QKV
               linear, RMSNorm), one replica per rank.

After timing, rank 0 checks the timed runs' outputs against the oracle (the CPU
restatement of the path, used here only as the checker): sampled heads of the
attention step (gathered from the ranks that own them over NCCL), sampled rows of
the GEMM (every rank's column block gathered), sampled rows of two long GQA heads,
and sampled rows of one block sequence.  Every input is generated from a global
seed per unit (head, KV group, weight), so the data do not depend on the number of
ranks.  The worst norm-wise relative error is printed as "max_rel_err".

`--impl reference` times the reference's CPU path for this op (the oracle: the
reference itself has no numeric implementation) on rank 0 with all host threads.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

B, H, S, D = 8, 32, 4096, 128
FWD_FLOPS = 2.0 * B * H * S * S * D          # causal forward
BWD_FLOPS = 2.5 * FWD_FLOPS
STEP_FLOPS = FWD_FLOPS + BWD_FLOPS
GEMM_N = 4096
METRIC = "causal attn fwd+bwd TFLOP/s & % bf16 peak at 1/2/4/8 B200; GEMM TFLOP/s"
CONFIG = {"workload": "bf16 causal attention fwd+bwd B=8 H=32 S=4096 D=128, heads sharded across ranks",
          "batch": B, "heads": H, "seq_len": S, "head_dim": D, "causal": True,
          "parallelism": "heads sharded, no collective on the hot path",
          "l2": "inputs larger than L2 (1 GiB per GPU at N=1; 128 MiB of inputs + outputs per GPU at N=8)"}
# FLOPs the backward kernels execute per head, in products of 2*S^2*D/2 (causal) each:
# k_attn_bwd_dkdv computes S^T, dP^T, dV and dK (4 products, 2x the forward),
# k_attn_bwd_dq computes S, dP and dQ (3 products, 1.5x the forward).
DKDV_FLOPS = 2.0 * FWD_FLOPS
DQ_FLOPS = 1.5 * FWD_FLOPS
# k_attn_bwd_dkdv DRAM traffic per launch from the ncu capture summarised in
# profiles/k_attn_bwd_dkdv_h32s4096.md (B*H=32 heads captured, scaled by the head count).
DKDV_TRAFFIC_PER_HEAD = (135.5e6 + 39.3e6) / 32

# pre-norm Llama block forward
BLK_B, BLK_S, BLK_DM, BLK_H, BLK_D, BLK_F = 4, 2048, 4096, 32, 128, 14336
BLK_T = BLK_B * BLK_S
BLK_FLOPS = (2.0 * BLK_T * BLK_DM * 3 * BLK_H * BLK_D        # QKV projection
             + 2.0 * BLK_T * BLK_H * BLK_D * BLK_DM          # output projection
             + 2.0 * BLK_T * BLK_DM * 2 * BLK_F              # gate + up
             + 2.0 * BLK_T * BLK_F * BLK_DM                  # down
             + 2.0 * BLK_B * BLK_H * BLK_S * BLK_S * BLK_D)  # causal attention (QK^T and PV, half)
# long-context grouped-query forward
GQA_HQ, GQA_HKV, GQA_S, GQA_D = 64, 8, 32768, 128
GQA_FLOPS = 2.0 * GQA_HQ * GQA_S * GQA_S * GQA_D
E2E_CHUNKS = 8  # head chunks of the pipelined end-to-end step


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["beacon", "reference"], default="beacon")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-block", action="store_true")
    ap.add_argument("--no-gqa", action="store_true")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 1590.0, 1400.0, "fallback"


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock / throttle-reason sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.device_id = device_id
        self.proc = None
        self.path = None

    def start(self):
        import tempfile
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.device_id], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                    power.append(float(parts[3]))
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        # samples under load: the upper half by power draw
        pw_med = statistics.median(power)
        loaded = [c for c, p in zip(sm, power) if p >= pw_med] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- distributed

def parse_cpulist(text):
    """'0-3,8,10-11' -> {0, 1, 2, 3, 8, 10, 11}."""
    cpus = set()
    for part in text.strip().split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        elif part:
            cpus.add(int(part))
    return cpus


def bind_host_threads(local):
    """With several ranks on one host, keeps this rank's threads on the CPUs that the host
    lists as local to its GPU (the PCI device's local_cpulist), so the pinned host buffers
    it allocates afterwards sit in the memory the GPU's copy engines reach without crossing
    between sockets.  Returns the CPU list used, or None where there is nothing to narrow."""
    import torch
    try:
        p = torch.cuda.get_device_properties(local)
        bus = "%04x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            text = f.read().strip()
        cur = os.sched_getaffinity(0)
        use = parse_cpulist(text) & cur
    except Exception:  # no CUDA device, no sysfs entry, an unparsable list: leave the threads as they are
        return None
    if not use or use == cur:
        return None
    os.sched_setaffinity(0, use)
    return text


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cpus = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        cpus = bind_host_threads(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local, cpus


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------------------- CPU baseline

def cpu_attention_sample(n_heads_max=None):
    """Time the oracle's attention fwd+bwd on a bounded sample of heads (all host threads)."""
    import oracle as O
    nthreads = O.num_threads()
    nh = min(nthreads if n_heads_max is None else n_heads_max, B * H)
    q = O.normal((1, nh, S, D), 2)
    k = O.normal((1, nh, S, D), 2, offset=q.size)
    v = O.normal((1, nh, S, D), 2, offset=2 * q.size)
    do = O.normal((1, nh, S, D), 2, offset=3 * q.size)
    t0 = time.perf_counter()
    _, lse = O.attention_fwd(q, k, v)
    O.attention_bwd(do, q, k, v, lse)
    dt = time.perf_counter() - t0
    flops = STEP_FLOPS * nh / (B * H)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": nthreads, "kind": "port",
            "sample": f"{nh} of {B * H} heads (S={S}, D={D}) fwd+bwd, float64-accumulating C oracle, "
                      f"{dt:.2f} s"}, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps_t = []
    info = None
    for i in range(args.warmup + args.steps):
        info, dt = cpu_attention_sample()
        if i >= args.warmup:
            steps_t.append(dt)
    ms = 1e3 * statistics.mean(steps_t)
    line = {"metric": METRIC, "value": info["value"], "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (f64 accumulation)", "data": "synthetic", "config": CONFIG,
            "impl": "reference", "cpu_baseline": info,
            "e2e": {"value": info["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- inputs and checks

ATTN_SEED, GEMM_SEED, BLOCK_SEED, GQA_SEED, BLOCK_BWD_SEED = 2, 1, 3, 4, 5
CHECK_TOL = 2e-2  # bf16 inputs, fp32 accumulation, gradients included (norm-wise)


def attn_head_inputs(t, h0, nh, dev):
    """Tensor t (0 Q, 1 K, 2 V, 3 dO) of global heads h0 .. h0+nh-1: [1, nh, S, D] bf16,
    each head N(0, 1) from its own generator."""
    import torch
    from beacon_b200.shard import unit_generator
    out = torch.empty(1, nh, S, D, dtype=torch.bfloat16, device=dev)
    for i in range(nh):
        g = unit_generator(ATTN_SEED, 4 * (h0 + i) + t, dev)
        out[0, i] = torch.randn(S, D, generator=g, device=dev).to(torch.bfloat16)
    return out


def check_attention(world, h0, nh, out, lse, dq, dk, dv, dev):
    """Heads 0 and B*H-1 of the timed step (gathered from their owners) against the oracle:
    out, lse, dq, dk, dv over every query and key row of each head.  Rank 0 returns
    {quantity: worst relative error}; the other ranks None."""
    import numpy as np
    import torch
    from beacon_b200.shard import gather_units
    wanted = [0, B * H - 1]
    got = {name: gather_units(t[0], h0, B * H, wanted, world).float().cpu().numpy()
           for name, t in (("out", out), ("lse", lse), ("dq", dq), ("dk", dk), ("dv", dv))}
    if h0 != 0:
        return None
    import oracle as O
    errs = {"out": 0.0, "lse": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    for i, gh in enumerate(wanted):
        qh, kh, vh, doh = (attn_head_inputs(t, gh, 1, dev)[0, 0].float().cpu().numpy() for t in range(4))
        ro, rl = O.attention_fwd_rows(qh, kh, vh, np.arange(S))
        rq, rk, rv = O.attention_bwd_head(doh, qh, kh, vh, rl)
        for name, r in (("out", ro), ("lse", rl), ("dq", rq), ("dk", rk), ("dv", rv)):
            errs[name] = max(errs[name], O.rel_err(got[name][i], r))
    return {"heads": wanted, **errs}


# --------------------------------------------------------------------------- GPU arm

def run_beacon(args, rank, world, local, cpus=None):
    import torch
    from beacon_b200 import ops

    if (B * H) % world != 0:
        raise SystemExit(f"{B * H} heads do not shard over {world} ranks")
    nh = B * H // world
    h0 = rank * nh  # first global (b*H + h) head of this rank
    dev = torch.device("cuda", local)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = str(local)
    burst, sustained, peak_kind = peaks()

    # inputs: head gh's Q, K, V, dO come from seed 2 and gh alone (the global tensors do not
    # depend on the rank count); pinned host copies feed the e2e step
    q, k, v, do = (attn_head_inputs(t, h0, nh, dev) for t in range(4))
    host = [t.cpu().pin_memory() for t in (q, k, v, do)]
    out = torch.empty_like(q)
    lse = torch.empty(1, nh, S, dtype=torch.float32, device=dev)
    L = ops._lib.lib()
    stream = torch.cuda.current_stream(dev)
    sp = ops._stream()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def step():
        ops.check(L.beacon_attention_adjoint_fwd(ops._p(out), ops._p(q), ops._p(k), ops._p(v), ops._p(lse), 1, nh,
                                                 S, D, 1, ops._lib.BF16, sp))
        ops.check(L.beacon_attention_adjoint_bwd(ops._p(dq), ops._p(dk), ops._p(dv), ops._p(do), ops._p(q),
                                                 ops._p(k), ops._p(v), ops._p(lse), 1, nh, S, D, 1, ops._lib.BF16,
                                                 None, 0, sp))

    def step_with_out():
        ops.check(L.beacon_attention_adjoint_fwd(ops._p(out), ops._p(q), ops._p(k), ops._p(v), ops._p(lse), 1, nh,
                                                 S, D, 1, ops._lib.BF16, sp))
        ops.check(L.beacon_attention_bwd_with_out(ops._p(dq), ops._p(dk), ops._p(dv), ops._p(do), ops._p(q),
                                                  ops._p(k), ops._p(v), ops._p(out), ops._p(lse), 1, nh, nh, S, D, 1,
                                                  ops._lib.BF16, None, 0, sp))

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return e0.elapsed_time(e1) / steps

    # ---- headline: drop-in fwd + bwd, device-resident.  The clock sampler starts
    # before the warm-up so that its first samples (nvidia-smi needs ~0.1 s to start)
    # already fall under load, and runs until the timed steps end.
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.profile_reset()
    ops.profile_enable(True)
    n0 = ops.launch_count()
    ms_local = timed(step, args.steps, 0)
    n_launch = ops.launch_count() - n0
    ops.profile_enable(False)
    clk = clocks.stop()
    bwd_ms, bwd_n = ops.profile_read("k_attn_bwd_dkdv")
    dq_ms, dq_n = ops.profile_read("k_attn_bwd_dq")
    fwd_ms, fwd_n = ops.profile_read("k_attn_fwd_tc")
    ms = max_over_ranks(ms_local, world)
    value = STEP_FLOPS / (ms * 1e-3) / 1e12

    # roofline of the dominant kernel: k_attn_bwd_dkdv, the FLOPs it executes per launch
    bwd_avg_ms = bwd_ms / max(bwd_n, 1)
    bwd_flops_local = DKDV_FLOPS * nh / (B * H)
    achieved = bwd_flops_local / (bwd_avg_ms * 1e-3) / 1e12
    traffic = None if DKDV_TRAFFIC_PER_HEAD is None else DKDV_TRAFFIC_PER_HEAD * nh
    dq_avg_ms = dq_ms / max(dq_n, 1)
    roofline = {"kernel": "k_attn_bwd_dkdv", "bound": "tensor", "achieved": achieved, "peak": burst,
                "unit": "TFLOP/s", "frac": achieved / burst, "traffic": traffic,
                "peak_kind": f"{peak_kind} bf16_tflops (burst: the timed region is well under a second)",
                "frac_of_sustained_peak": achieved / sustained, "sustained_peak": sustained,
                "avg_launch_ms": bwd_avg_ms, "launches": bwd_n,
                "dq_kernel": {"kernel": "k_attn_bwd_dq", "avg_launch_ms": dq_avg_ms,
                              "tflops_executed": DQ_FLOPS * nh / (B * H) / (dq_avg_ms * 1e-3) / 1e12},
                "fwd_kernel": {"kernel": "k_attn_fwd_tc", "avg_launch_ms": fwd_ms / max(fwd_n, 1),
                               "launches_per_step": fwd_n / max(args.steps, 1)}}

    # ---- the timed step's outputs (deterministic: every step writes the same values)
    check_attn = check_attention(world, h0, nh, out, lse, dq, dk, dv, dev)

    # ---- with_out variant
    ms_wo = max_over_ranks(timed(step_with_out, args.steps, 2), world)
    with_out = {"value": STEP_FLOPS / (ms_wo * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_wo,
                "note": "backward given the forward output (beacon_attention_bwd_with_out), no recompute"}

    # ---- e2e: pinned host -> device, fwd+bwd, device -> host of out, dq, dk, dv.  The
    # heads are independent, so each step runs as E2E_CHUNKS head chunks on three streams:
    # chunk c's host->device copies, its fwd+bwd, and its device->host copies overlap the
    # neighbouring chunks' (PCIe carries both directions at once).  Every byte of every
    # step still crosses PCIe inside the timed region.
    e2e = None
    if not args.no_e2e:
        host_out = [torch.empty(1, nh, S, D, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
        h2d = sum(h.numel() * h.element_size() for h in host)
        d2h = sum(h.numel() * h.element_size() for h in host_out)
        n_chunks = max(1, min(E2E_CHUNKS, nh))
        bounds = [(c * nh // n_chunks, (c + 1) * nh // n_chunks) for c in range(n_chunks)]
        s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        cmp_handle = ctypes.c_void_p(s_cmp.cuda_stream)
        ev_in = [torch.cuda.Event() for _ in range(n_chunks)]
        ev_cmp = [torch.cuda.Event() for _ in range(n_chunks)]
        ev_out = [torch.cuda.Event() for _ in range(n_chunks)]
        started = [False] * n_chunks

        def chunk_call(h0, h1):
            hc = h1 - h0
            sl = lambda t: ops._p(t[:, h0:h1])
            ops.check(L.beacon_attention_adjoint_fwd(sl(out), sl(q), sl(k), sl(v), sl(lse), 1, hc, S, D, 1,
                                                     ops._lib.BF16, cmp_handle))
            ops.check(L.beacon_attention_adjoint_bwd(sl(dq), sl(dk), sl(dv), sl(do), sl(q), sl(k), sl(v), sl(lse),
                                                     1, hc, S, D, 1, ops._lib.BF16, None, 0, cmp_handle))

        def e2e_step():
            for c, (h0, h1) in enumerate(bounds):
                with torch.cuda.stream(s_in):
                    if started[c]:
                        s_in.wait_event(ev_cmp[c])  # the previous step's compute has read chunk c
                    for dst, src in zip((q, k, v, do), host):
                        dst[:, h0:h1].copy_(src[:, h0:h1], non_blocking=True)
                    ev_in[c].record(s_in)
                s_cmp.wait_event(ev_in[c])
                if started[c]:
                    s_cmp.wait_event(ev_out[c])  # the previous step's results of chunk c are out
                chunk_call(h0, h1)
                ev_cmp[c].record(s_cmp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_cmp[c])
                    for dst, src in zip(host_out, (out, dq, dk, dv)):
                        dst[:, h0:h1].copy_(src[:, h0:h1], non_blocking=True)
                    ev_out[c].record(s_out)
                started[c] = True

        def timed_e2e(steps, warmup):
            for _ in range(warmup):
                e2e_step()
            torch.cuda.synchronize()
            barrier(world)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s_in)
            s_cmp.wait_event(e0)
            s_out.wait_event(e0)
            for _ in range(steps):
                e2e_step()
            s_out.wait_stream(s_cmp)
            s_out.wait_stream(s_in)
            e1.record(s_out)
            torch.cuda.synchronize()
            barrier(world)
            return e0.elapsed_time(e1) / steps

        ms_e2e = max_over_ranks(timed_e2e(max(2, args.steps // 2), 1), world)
        e2e = {"value": STEP_FLOPS / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": int(sum_over_ranks(h2d, world)),
               "d2h_bytes_per_step": int(sum_over_ranks(d2h, world)),
               "api": f"beacon_attention_adjoint_fwd + beacon_attention_adjoint_bwd on {n_chunks} head chunks, "
                      "copies in, compute and copies out overlapped on three streams",
               "host_cpus": (f"each rank's threads on its GPU's local CPUs (rank 0: {cpus})" if cpus
                             else "not narrowed")}

    del q, k, v, do, out, dq, dk, dv, host
    torch.cuda.empty_cache()

    # ---- GEMM 4096^3, columns of B sharded
    gemm = None
    check_gemm = None
    if not args.no_gemm:
        from beacon_b200.shard import gather_rows, unit_generator
        ncols = GEMM_N // world
        # A and B entries U(-1, 1) from the GEMM seed (A: unit 0, B: unit 1); every rank
        # holds A and its own column block of B
        a = (torch.rand(GEMM_N, GEMM_N, generator=unit_generator(GEMM_SEED, 0, dev), device=dev) * 2 - 1
             ).to(torch.bfloat16)
        b_full = (torch.rand(GEMM_N, GEMM_N, generator=unit_generator(GEMM_SEED, 1, dev), device=dev) * 2 - 1
                  ).to(torch.bfloat16)
        bm = b_full[:, rank * ncols:(rank + 1) * ncols].contiguous()
        c = torch.empty(GEMM_N, ncols, dtype=torch.bfloat16, device=dev)
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        for _ in range(3):
            ops.matmul_fwd(a, bm, out=c)
        torch.cuda.synchronize()
        barrier(world)
        times = []
        for _ in range(max(args.steps, 5)):
            flush.fill_(1)  # evict A, B, C from the 126 MB L2
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ops.matmul_fwd(a, bm, out=c)
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        barrier(world)
        gms = max_over_ranks(statistics.median(times), world)
        gt = 2.0 * GEMM_N ** 3 / (gms * 1e-3) / 1e12
        gemm = {"value": gt, "unit": "TFLOP/s", "ms": gms, "frac_of_burst_peak": gt / burst / world,
                "config": f"bf16 {GEMM_N}^3, B columns sharded {world}-way, L2 flushed between iterations",
                "per_gpu_tflops": gt / world,
                # the shard's tile shape as the library chose it: at 8 ranks the 4096 x 512 shard
                # has too few tiles to fill the SMs, and the launch's fixed cost weighs more
                "shard_plan": dict(ops.matmul_plan(GEMM_N, GEMM_N, ncols), shard=[GEMM_N, ncols, GEMM_N])}
        # 16 sampled rows of C: every rank's column block gathered to rank 0
        rows = torch.arange(0, GEMM_N, GEMM_N // 16, device=dev)
        c_rows = gather_rows(c[rows].t().contiguous(), world).t()  # [16, GEMM_N]
        if rank == 0:
            import oracle as O
            ref = O.matmul_fwd(a[rows].float().cpu().numpy(), b_full.float().cpu().numpy())
            check_gemm = {"rows": 16, "c": O.rel_err(c_rows.float().cpu().numpy(), ref)}
        # the same GEMM with fp8 e4m3 weights (fp32 master quantised per tensor on the device,
        # decoded inside the GEMM pipeline, the scale read on the device)
        w8, wscale, _ = ops.quantize_fp8e4m3(b_full[:, rank * ncols:(rank + 1) * ncols].float().contiguous())
        c8 = torch.empty_like(c)
        times8 = []
        for i in range(max(args.steps, 5) + 3):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ops.linear_fp8w_fwd_devscale(a, w8, wscale, out=c8)
            e1.record(stream)
            e1.synchronize()
            if i >= 3:
                times8.append(e0.elapsed_time(e1))
        barrier(world)
        g8ms = max_over_ranks(statistics.median(times8), world)
        gemm["fp8_weights"] = {"value": 2.0 * GEMM_N ** 3 / (g8ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": g8ms,
                               "api": "beacon_quantize_fp8e4m3 then beacon_linear_fp8w_fwd_devscale "
                                      "(k_gemm_fp8w_tc2: e4m3 decoded inside the GEMM pipeline)"}
        if rank == 0:
            import oracle as O
            wq = (O.from_fp8_bits(w8.cpu().numpy()) * float(wscale.item())).astype("float32")
            ref8 = O.matmul_fwd(a[rows].float().cpu().numpy(), wq)
            check_gemm["c_fp8_weights_local_columns"] = O.rel_err(c8[rows].float().cpu().numpy(), ref8)
        del a, bm, b_full, c, flush, w8, c8

    block, check_block = (None, None) if args.no_block else bench_block(args, rank, world, dev, stream)
    gqa, check_gqa = (None, None) if args.no_gqa else bench_gqa(args, rank, world, dev, stream)
    block_bwd, check_block_bwd = (None, None) if args.no_block else bench_block_bwd(args, rank, world, dev, stream)

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu, _ = cpu_attention_sample()
    checks = {"attention": check_attn, "gemm": check_gemm, "gqa": check_gqa, "block": check_block,
              "block_backward": check_block_bwd}
    worst = 0.0
    for c in checks.values():
        if c:
            worst = max([worst] + [float(x) for k_, x in c.items() if isinstance(x, float)])
    max_rel_err = {"value": worst, "tolerance": CHECK_TOL, "ok": worst <= CHECK_TOL,
                   "measure": "max |x - ref| / max |ref| per checked tensor, oracle on sampled units", **checks}
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic: i.i.d. N(0,1) Q/K/V/dO, seeded per head",
            "config": CONFIG, "frac_of_peak": value / (burst * world),
            "frac_of_sustained_peak": value / (sustained * world),
            "roofline": roofline, "max_rel_err": max_rel_err, "cpu_baseline": cpu, "e2e": e2e,
            "with_out": with_out, "gemm": gemm, "block": block, "block_backward": block_bwd, "gqa": gqa,
            "clocks": clk, "gpu_launches": int(n_launch), "impl": "beacon"}
    print(json.dumps(line), flush=True)


def _time_calls(fn, stream, iters, warmup):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def bench_block(args, rank, world, dev, stream):
    """One pre-norm Llama block forward per rank (replicas), weights N(0, 0.02), x N(0, 1)."""
    import torch
    from beacon_b200 import ops
    from beacon_b200.shard import unit_generator

    def w(unit, *shape, std=0.02):
        return (torch.randn(*shape, generator=unit_generator(BLOCK_SEED, unit, dev), device=dev) * std
                ).to(torch.bfloat16)

    x = w(0, BLK_T, BLK_DM, std=1.0)
    n1 = torch.ones(BLK_DM, device=dev, dtype=torch.bfloat16)
    n2 = torch.ones(BLK_DM, device=dev, dtype=torch.bfloat16)
    wqkv, wo = w(1, BLK_DM, 3 * BLK_H * BLK_D), w(2, BLK_H * BLK_D, BLK_DM)
    wg, wu, wd = w(3, BLK_DM, BLK_F), w(4, BLK_DM, BLK_F), w(5, BLK_F, BLK_DM)
    out = torch.empty_like(x)
    ws = torch.empty(ops.llama_block_workspace_bytes(BLK_B, BLK_S, BLK_DM, BLK_H, BLK_H, BLK_D, BLK_F),
                     dtype=torch.uint8, device=dev)

    def fn():
        ops.llama_block_fwd(x, n1, wqkv, wo, n2, wg, wu, wd, BLK_B, BLK_S, BLK_H, BLK_H, out=out, workspace=ws)

    # the norms folded into the GEMMs after them: gains folded into the weights once per
    # weight version, outside the timed region
    wqkv_f, wg_f, wu_f = ops.llama_block_fold_weights(n1, wqkv, n2, wg, wu)
    out_f = torch.empty_like(x)

    def fn_folded():
        ops.llama_block_fwd_folded(x, wqkv_f, wo, wg_f, wu_f, wd, BLK_B, BLK_S, BLK_H, BLK_H, out=out_f,
                                   workspace=ws)

    # the two forms alternate call by call (each pair in the other order than the one
    # before), every call timed by its own events, and each form keeps its median: under the
    # 1 kW power cap the clock falls by 10-20% as the GPU warms over the few seconds of the
    # run, more than the forms differ, and this way both forms see the same trend (timing
    # them in alternating rounds and keeping each one's fastest round favoured whichever form
    # came first in the first round)
    pairs = max(10, args.steps // 2)
    for f in (fn, fn_folded, fn, fn_folded):
        f()
    torch.cuda.synchronize()
    barrier(world)
    ev = {"un": [], "fo": []}
    for i in range(pairs):
        for name, f in ((("un", fn), ("fo", fn_folded)) if i % 2 == 0 else (("fo", fn_folded), ("un", fn))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            f()
            e1.record(stream)
            ev[name].append((e0, e1))
    torch.cuda.synchronize()
    t_un = [a.elapsed_time(b) for a, b in ev["un"]]
    t_fo = [a.elapsed_time(b) for a, b in ev["fo"]]
    ms = max_over_ranks(statistics.median(t_un), world)
    ms_f = max_over_ranks(statistics.median(t_fo), world)
    torch.cuda.synchronize()
    check = None
    if rank == 0:  # rows of sequence 1 of both timed replicas against the sampled-row block oracle
        import numpy as np
        import oracle as O
        seq = 1
        rows = np.array([0, 1, 127, 128, 777, 1500, BLK_S - 2, BLK_S - 1])
        h = lambda t: t.float().cpu().numpy()
        xs = h(x[seq * BLK_S:(seq + 1) * BLK_S])
        ones = np.ones(BLK_DM, dtype=np.float32)
        ref = O.llama_block_fwd_rows(xs, ones, h(wqkv), h(wo), ones, h(wg), h(wu), h(wd), BLK_H, BLK_H, rows)
        ridx = torch.from_numpy(rows).to(dev)
        got, got_f = h(out[seq * BLK_S + ridx]), h(out_f[seq * BLK_S + ridx])
        check = {"sequence": seq, "rows": rows.tolist(), "out": O.rel_err(got, ref),
                 "branch": O.rel_err(got - xs[rows], ref - xs[rows]), "out_folded": O.rel_err(got_f, ref),
                 "branch_folded": O.rel_err(got_f - xs[rows], ref - xs[rows])}
    del x, wqkv, wo, wg, wu, wd, out, ws, wqkv_f, wg_f, wu_f, out_f
    torch.cuda.empty_cache()
    return {"value": BLK_FLOPS * world / (ms_f * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms_f,
            "per_gpu_tflops": BLK_FLOPS / (ms_f * 1e-3) / 1e12, "flops_per_block": BLK_FLOPS,
            "config": f"pre-norm Llama block forward, batch {BLK_B} x seq {BLK_S}, d_model {BLK_DM}, "
                      f"{BLK_H} x {BLK_D} heads, SwiGLU {BLK_F}, bf16; one replica per rank",
            "api": "beacon_llama_block_fwd_folded (RMSNorms folded into the GEMMs: 6 launches + a memset)",
            "unfused": {"ms": ms, "per_gpu_tflops": BLK_FLOPS / (ms * 1e-3) / 1e12,
                        "api": "beacon_llama_block_fwd (RMSNorm kernels write normalised rows: 7 launches)"}}, check


def bench_block_bwd(args, rank, world, dev, stream):
    """The backward operators at the block's shapes, one replica per rank: swiglu_bwd
    (mlp.rs:31-52), linear_bwd of the QKV projection (matmul.rs:60-78) and rmsnorm_bwd
    (norm.rs:33-50) at tokens 8192, d_model 4096, SwiGLU hidden 14336, QKV width 12288.
    Algorithmic FLOPs: the SwiGLU backward 12 T d F (dWd, dh, dWg, dWu, dx; its recompute of
    gate and up is not counted), the linear backward 4 T d N; the RMSNorm backward is
    reported in GB/s of x, dy read and dx written."""
    import torch
    from beacon_b200 import ops
    from beacon_b200.shard import unit_generator
    T, dm, F, N = BLK_T, BLK_DM, BLK_F, 3 * BLK_H * BLK_D

    def w(unit, *shape, std=0.02):
        return (torch.randn(*shape, generator=unit_generator(BLOCK_BWD_SEED, unit, dev), device=dev) * std
                ).to(torch.bfloat16)

    x, dy = w(0, T, dm, std=1.0), w(1, T, dm, std=1.0)
    wg, wu, wd = w(2, dm, F), w(3, dm, F), w(4, F, dm)
    wqkv, dqkv = w(5, dm, N), w(6, T, N, std=1.0)
    g = (1.0 + w(7, dm, std=0.1).float()).to(torch.bfloat16)
    _, rms = ops.rmsnorm_fwd(x, g)
    L, sp, P, bf = ops._lib.lib(), ops._stream(), ops._p, ops._lib.BF16
    sdx, sdg, sdu, sdd = torch.empty_like(x), torch.empty_like(wg), torch.empty_like(wu), torch.empty_like(wd)
    sw_ws = torch.empty(ops._lib.lib().beacon_swiglu_workspace_size(T, dm, F, bf, 1), dtype=torch.uint8, device=dev)
    ldx, ldw, ldb = torch.empty_like(x), torch.empty_like(wqkv), torch.empty(N, dtype=torch.bfloat16, device=dev)
    rdx, rdg = torch.empty_like(x), torch.empty_like(g)

    def swiglu():
        ops.check(L.beacon_swiglu_adjoint_bwd(P(sdx), P(sdg), P(sdu), P(sdd), P(dy), P(x), P(wg), P(wu), P(wd), T, dm,
                                              F, bf, P(sw_ws), sw_ws.numel(), sp))

    def linear():
        ops.check(L.beacon_linear_bwd(P(ldx), P(ldw), P(ldb), P(dqkv), P(x), P(wqkv), T, dm, N, bf, sp))

    def rmsnorm():
        ops.check(L.beacon_rmsnorm_adjoint_bwd(P(rdx), P(rdg), P(dy), P(x), P(rms), P(g), T, dm, bf, None, 0, sp))

    iters = max(10, args.steps // 2)
    barrier(world)
    res = {}
    for name, fn in (("swiglu", swiglu), ("linear", linear), ("rmsnorm", rmsnorm)):
        res[name] = max_over_ranks(min(_time_calls(fn, stream, iters, 2) for _ in range(2)), world)
    torch.cuda.synchronize()
    check = None
    if rank == 0:  # sampled rows of dx and columns of the weight gradients against the oracle
        import numpy as np
        import oracle as O
        rng = np.random.default_rng(BLOCK_BWD_SEED)
        rows = np.sort(rng.choice(T, 16, replace=False))
        cols = np.sort(rng.choice(F, 16, replace=False))
        h = lambda t: t.float().cpu().numpy()
        hx, hdy = h(x), h(dy)
        rs = O.swiglu_bwd_sampled(hdy, hx, h(wg), h(wu), h(wd), rows, cols)
        f64 = lambda a: np.asarray(a, dtype=np.float64)
        lcols = np.sort(rng.choice(N, 16, replace=False))
        hdq, hw = h(dqkv), h(wqkv)
        rr = torch.from_numpy(rows).to(dev)
        ndx, ndg = O.rmsnorm_bwd(hdy, hx, h(rms), h(g))
        check = {"rows": rows.tolist(), "swiglu_dx": O.rel_err(h(sdx[rr]), rs[0]),
                 "swiglu_dwg": O.rel_err(h(sdg)[:, cols], rs[1]), "swiglu_dwu": O.rel_err(h(sdu)[:, cols], rs[2]),
                 "swiglu_dwd": O.rel_err(h(sdd)[cols, :], rs[3]),
                 "linear_dx": O.rel_err(h(ldx[rr]), f64(hdq[rows]) @ f64(hw).T),
                 "linear_dw": O.rel_err(h(ldw)[:, lcols], f64(hx).T @ f64(hdq[:, lcols])),
                 "linear_db": O.rel_err(h(ldb), f64(hdq).sum(axis=0)),
                 "rmsnorm_dx": O.rel_err(h(rdx), ndx), "rmsnorm_dweight": O.rel_err(h(rdg), ndg)}
    del x, dy, wg, wu, wd, wqkv, dqkv, sdx, sdg, sdu, sdd, sw_ws, ldx, ldw, ldb, rdx, rdg
    torch.cuda.empty_cache()
    sw_fl, li_fl, rn_b = 12.0 * T * dm * F, 4.0 * T * dm * N, 3.0 * T * dm * 2 + 4.0 * T
    return {"config": f"tokens {T}, d_model {dm}, SwiGLU hidden {F}, QKV width {N}, bf16; one replica per rank",
            "swiglu_bwd": {"ms": res["swiglu"], "per_gpu_tflops": sw_fl / (res["swiglu"] * 1e-3) / 1e12,
                           "api": "beacon_swiglu_adjoint_bwd (5 GEMMs)"},
            "linear_bwd": {"ms": res["linear"], "per_gpu_tflops": li_fl / (res["linear"] * 1e-3) / 1e12,
                           "api": "beacon_linear_bwd (dx, dW, dbias)"},
            "rmsnorm_bwd": {"ms": res["rmsnorm"], "per_gpu_gbs": rn_b / (res["rmsnorm"] * 1e-3) / 1e9,
                            "api": "beacon_rmsnorm_adjoint_bwd (row kernel + column sum)"}}, check


def bench_gqa(args, rank, world, dev, stream):
    """Causal GQA forward, S=32768; the 8 KV groups (8 query heads each) sharded across ranks."""
    import torch
    from beacon_b200 import ops
    from beacon_b200.shard import gather_units, unit_generator
    if GQA_HKV % world != 0:
        return None, None
    hkv = GQA_HKV // world
    grp = GQA_HQ // GQA_HKV
    hq = hkv * grp
    kv0, q0 = rank * hkv, rank * hkv * grp  # first global KV head / query head of this rank

    def gen(unit, n):  # n heads [1, n, S, D], head i from unit + i
        t = torch.empty(1, n, GQA_S, GQA_D, dtype=torch.bfloat16, device=dev)
        for i in range(n):
            t[0, i] = torch.randn(GQA_S, GQA_D, generator=unit_generator(GQA_SEED, unit + i, dev),
                                  device=dev).to(torch.bfloat16)
        return t

    # units: query head h -> h, KV head g -> GQA_HQ + g (K), GQA_HQ + GQA_HKV + g (V)
    q = gen(q0, hq)
    k = gen(GQA_HQ + kv0, hkv)
    v = gen(GQA_HQ + GQA_HKV + kv0, hkv)
    out = torch.empty_like(q)
    lse = torch.empty(1, hq, GQA_S, dtype=torch.float32, device=dev)
    L = ops._lib.lib()
    sp = ops._stream()

    def fn():
        ops.check(L.beacon_attention_gqa_fwd(ops._p(out), ops._p(q), ops._p(k), ops._p(v), ops._p(lse), 1, hq, hkv,
                                             GQA_S, GQA_D, 1, ops._lib.BF16, sp))

    barrier(world)
    ms = max_over_ranks(_time_calls(fn, stream, 10, 3), world)
    # query heads 0 and 63 (KV groups 0 and 7): the last 128 rows (all 256 key tiles deep)
    # and 128 rows spread over the sequence, gathered from their owners
    import numpy as np
    rows = np.unique(np.concatenate([np.linspace(0, GQA_S - 129, 128).astype(np.int64),
                                     np.arange(GQA_S - 128, GQA_S)]))
    ridx = torch.from_numpy(rows).to(dev)
    wanted = [0, GQA_HQ - 1]
    got = gather_units(out[0][:, ridx], q0, GQA_HQ, wanted, world).float().cpu().numpy()
    check = None
    if rank == 0:
        import oracle as O
        err = 0.0
        for i, h in enumerate(wanted):
            g = h // grp
            qh = gen(h, 1)[0, 0].float().cpu().numpy()
            kh = gen(GQA_HQ + g, 1)[0, 0].float().cpu().numpy()
            vh = gen(GQA_HQ + GQA_HKV + g, 1)[0, 0].float().cpu().numpy()
            ro, _ = O.attention_fwd_rows(qh, kh, vh, rows)
            err = max(err, O.rel_err(got[i], ro))
        check = {"query_heads": wanted, "rows": int(rows.size), "out": err}
    del q, k, v, out, lse
    torch.cuda.empty_cache()
    return {"value": GQA_FLOPS / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms,
            "per_gpu_tflops": GQA_FLOPS / world / (ms * 1e-3) / 1e12,
            "config": f"causal GQA forward B=1, {GQA_HQ} query / {GQA_HKV} KV heads, S={GQA_S}, D={GQA_D}, bf16; "
                      f"{hq} query heads ({hkv} KV groups) per rank",
            "api": "beacon_attention_gqa_fwd"}, check


def main():
    args = parse_args()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local, cpus = dist_setup(args.gpus)
    try:
        run_beacon(args, rank, world, local, cpus)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
