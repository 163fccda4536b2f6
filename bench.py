"""Benchmark of the fused radix decode + linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

One STEP is one decode token's linear stack at batch 1: every packed linear of
every layer through the fused decode + GEMV (row-sharded over N ranks with an
NCCL all-gather of each output slice when N > 1), replayed from one CUDA
graph. Weights are random-init N(0, 0.02) bf16 of the named architecture
packed with the `sip` profile by this package's encoder (byte-identical to the
reference's); activations N(0, 1) bf16. The stack (tens of GB) is far larger
than L2, so no flush is needed between steps.

Workloads:
  qwen3-32b   configs[3]: 64 layers, q 8192x5120, k/v 1024x5120, o 5120x8192,
              gate/up 25600x5120, down 5120x25600; row-sharded over N GPUs
              (the default at every N: the metric's 1/2/4/8-GPU config, and it
              fits one GPU)
  qwen3-8b    configs[1]: 36 layers of q/k/v/o 4096, gate/up 12288x4096, down
              4096x12288, plus the raw bf16 lm_head 151936x4096 (reported
              beside the headline at N = 1)

Rank 0 prints ONE JSON line. `--impl reference` times the reference's own CPU
path (its native decoder compiled from its sources into oracle/_ref, then
torch F.linear over the decoded weights: swap.py's "cpu" route) on the host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "qwen3-32b": dict(layers=64, hidden=5120, linears=[("q", 8192, 5120), ("k", 1024, 5120), ("v", 1024, 5120),
                                                        ("o", 5120, 8192), ("gate", 25600, 5120),
                                                        ("up", 25600, 5120), ("down", 5120, 25600)], head=None),
    "qwen3-8b": dict(layers=36, hidden=4096, linears=[("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096),
                                                       ("o", 4096, 4096), ("gate", 12288, 4096),
                                                       ("up", 12288, 4096), ("down", 4096, 12288)],
                     head=(151936, 4096)),
}
# the headline metric, printed alike by both arms (BASELINE.json "metric")
METRIC = "decode tokens/s @ batch 1 + fused decode-GEMV HBM GB/s (% of B200 peak), 1/2/4/8 GPU"
# which input each linear reads: the hidden state (the step's H2D input) or
# the attention / MLP intermediate (a resident synthetic activation)
HIDDEN_INPUT = {"q", "k", "v", "gate", "up"}
# linears that read the same activations run as ONE fused launch (one
# dm_tensor_create_multi handle each): q|k|v and gate|up
GROUPS = (("qkv", ("q", "k", "v")), ("o", ("o",)), ("gate_up", ("gate", "up")), ("down", ("down",)))


def groups_of(wl, fuse=True):
    """[(group name, [(linear, R, C), ...])] in step order."""
    lin = {n: (n, R, C) for n, R, C in WORKLOADS[wl]["linears"]}
    if not fuse:
        return [(n, [lin[n]]) for n, _, _ in WORKLOADS[wl]["linears"]]
    return [(g, [lin[n] for n in names]) for g, names in GROUPS]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="qwen3-32b")
    ap.add_argument("--no-fuse", action="store_true", help="one launch per linear instead of q|k|v and gate|up")
    ap.add_argument("--gather", choices=("peer", "nccl"), default="peer",
                    help="N > 1: the output gather fused into the GEMV over NVLink (peer), or NCCL all-gather")
    ap.add_argument("--launch", choices=("auto", "chain", "linear"), default="auto",
                    help="the step as one persistent launch over every linear (dm_chain_run), or one launch per "
                         "linear (the per-linear plugin route); auto: per-linear (measured faster at N = 1 and 4, "
                         "2.4 %% slower at N = 2); the other is timed beside it")
    ap.add_argument("--variants", type=int, default=2,
                    help="distinct random tensors per shape; every layer still gets its own HBM copy")
    ap.add_argument("--no-secondary", action="store_true", help="skip the qwen3-8b chain beside the headline")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS dense arm")
    ap.add_argument("--no-configs", action="store_true", help="skip configs 3 (gulp, M = 2/4/8) and 5 (prefill)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (small profiling cases only; the headline uses the model's)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """nvidia-smi samples of the SM clock and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # nvidia-smi takes a moment to start: wait for its first sample, so
        # that a short timed region (20 steps of a few ms at N = 8) is covered
        t0 = time.time()
        while time.time() - t0 < 10 and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        power = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(power) if power else None}


# --------------------------------------------------------------- weights --

def make_bits(R, C, seed, device):
    """N(0, 0.02) bf16 bits [R, C] drawn on the GPU from `seed`, as numpy."""
    import numpy as np
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn((R, C), generator=g, device=device) * 0.02).to(torch.bfloat16)
    return w.view(torch.int16).cpu().numpy().view(np.uint16)


def build_stack(wl, rank, world, device, variants, log, fuse=True):
    """Per layer and launch group: this rank's row shard of every linear of
    the group (a fused handle for q|k|v and gate|up), each layer in its own
    HBM (variants distinct random tensors per shape, cloned per layer).
    Returns (layers[[runtime]], pack stats)."""
    from drinkme_b200 import codec, shard, swap

    spec = WORKLOADS[wl]
    groups = groups_of(wl, fuse)
    stats = {}
    base = {}
    t0 = time.time()
    for v in range(variants):
        packs = {}
        for j, (name, R, C) in enumerate(spec["linears"]):
            bits = make_bits(R, C, seed=1000 * v + 17 * j + R + C, device=device)
            p = codec.pack_array_radix(bits, "sip")
            assert p is not None
            packs[name] = p
            stats[(name, v)] = {"bpw": p["bpw"], "words": int(p["rx_data"].size)}
            del bits
        for gname, parts in groups:
            ranges = [shard.row_range(R, rank, world) for _, R, _ in parts]
            if all(r1 <= r0 for r0, r1 in ranges):
                base[(gname, v)] = None
            elif len(parts) == 1:
                base[(gname, v)] = swap.to_device_radix(packs[parts[0][0]], device, *ranges[0])
            else:
                base[(gname, v)] = swap.to_device_radix_fused([packs[n] for n, _, _ in parts], device, ranges)
        del packs
    log(f"packed {len(stats)} distinct tensors into {len(base)} launch groups in {time.time() - t0:.1f}s")
    layers = []
    for layer in range(spec["layers"]):
        row = []
        for gname, _ in groups:
            rt = base[(gname, layer % variants)]
            if rt is not None and layer >= variants:
                rt = dict(rt, rx_handle=rt["rx_handle"].clone())
            row.append(rt)
        layers.append(row)
    log(f"stack resident after {time.time() - t0:.1f}s")
    return layers, stats


# ------------------------------------------------------------------- step --

class Chain:
    """One decode token's linear stack with static buffers, for graph capture:
    per layer, one launch per group (q|k|v, o, gate|up, down when fused)."""

    def __init__(self, wl, layers, rank, world, device, head_weight=None, fuse=True, gather="peer", launch="linear"):
        import torch

        from drinkme_b200 import shard

        self.spec = WORKLOADS[wl]
        self.groups = groups_of(wl, fuse)
        self.layers = layers
        self.world = world
        self.device = device
        hidden = self.spec["hidden"]
        g = torch.Generator(device=device).manual_seed(12345)
        self.x_hidden = torch.randn((1, hidden), generator=g, device=device).to(torch.bfloat16)
        self.x_other = {}
        for _, parts in self.groups:
            name, R, C = parts[0]
            if name not in HIDDEN_INPUT and C not in self.x_other:
                self.x_other[C] = torch.randn((1, C), generator=g, device=device).to(torch.bfloat16)
        # per group: the gather slot of one rank (sum of the parts' largest shards)
        self.slot = [sum(shard.shard_rows_padded(R, world) for _, R, _ in parts) for _, parts in self.groups]
        self.outs, self.works = [], []
        for row in layers:
            o, w = [], []
            for gi, rt in enumerate(row):
                rows = 0 if rt is None else rt["R"]
                o.append(torch.zeros((1, self.slot[gi] if world > 1 else rows), dtype=torch.bfloat16,
                                     device=device))
                w.append(torch.empty((world, 1, self.slot[gi]), dtype=torch.bfloat16, device=device)
                         if world > 1 else None)
            self.outs.append(o)
            self.works.append(w)
        self.head = head_weight
        self.head_out = None
        self.last = None
        self.gather = gather if world > 1 else None
        self.plan = None
        self.persistent = None
        if launch == "chain":
            # every linear of the step in one persistent launch; link k waits
            # for link k - 1 (the previous launch's last for link 0), as each
            # linear of a decode step waits for its predecessor's output
            from drinkme_b200 import shard as _shard

            if any(rt is None for row in layers for rt in row):
                raise ValueError("the chain needs rows of every linear on every rank")
            G = len(self.groups)
            n = len(layers) * G
            self.plan = _shard.PeerGather([self.slot[i % G] if world > 1 else layers[i // G][i % G]["R"]
                                           for i in range(n)], 1, torch.bfloat16, rank, world, device)
            self.persistent = self.plan.chain([(layers[k // G][k % G], self.inputs(k % G), k, (k - 1) % n, None)
                                               for k in range(n)])
            return
        if self.gather == "peer":
            from drinkme_b200 import shard as _shard

            if any(rt is None for row in layers for rt in row):
                raise ValueError("the fused gather needs rows of every linear on every rank")
            G = len(self.groups)
            self.plan = _shard.PeerGather([self.slot[i % G] for i in range(len(layers) * G)], 1, torch.bfloat16,
                                          rank, world, device)

    def close(self):
        if self.persistent is not None:
            self.persistent.close()
            self.persistent = None
        if self.plan is not None:
            self.plan.close()
            self.plan = None

    def inputs(self, gi):
        name, _, C = self.groups[gi][1][0]
        return self.x_hidden if name in HIDDEN_INPUT else self.x_other[C]

    def launches_per_step(self):
        n = 1 if self.persistent is not None else sum(1 for row in self.layers for rt in row if rt is not None)
        return n + (1 if self.head is not None else 0)

    def step(self):
        """Every group's GEMV of every layer; with N ranks each output slice
        is all-gathered (rank-major: the consumer of q|k|v or gate|up reads
        rank k's rows of each part at a fixed offset of slot k)."""
        import torch
        import torch.distributed as dist

        from drinkme_b200 import radix_ops

        G = len(self.groups)
        n = len(self.layers) * G
        if self.persistent is not None:
            self.persistent.run()
            self.last = self.plan.output(n - 1)
            if self.head is not None:
                self.head_out = radix_ops.gemv_raw(self.head, self.x_hidden, None, torch.bfloat16)
                self.last = self.head_out
            return self.last
        for li, row in enumerate(self.layers):
            for gi, rt in enumerate(row):
                if self.plan is not None:
                    # this rank's rows into every rank's gathered output; wait
                    # for the previous linear's gather before reading x
                    i = li * G + gi
                    self.plan.gemv(rt, self.inputs(gi), i, wait=(i - 1) % n)
                    self.last = self.plan.output(i)
                    continue
                out = self.outs[li][gi]
                if rt is not None:
                    radix_ops.gemv_into(rt, self.inputs(gi), None, out[:, :rt["R"]])
                if self.world > 1:
                    work = self.works[li][gi]
                    dist.all_gather_into_tensor(work.view(self.world, self.slot[gi]), out.view(-1))
                    self.last = work
                else:
                    self.last = out
        if self.head is not None:
            self.head_out = radix_ops.gemv_raw(self.head, self.x_hidden, None, torch.bfloat16)
            self.last = self.head_out
        return self.last


def time_graph(chain, steps, warmup, world, rank, device, h2d=None):
    """CUDA-graph the step, replay `warmup` times, then time `steps` replays
    with events on the replay stream between barriers; max over ranks."""
    import torch
    import torch.distributed as dist

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(2):
            chain.step()  # first-call setup (kernel attributes, NCCL) outside capture
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        out = chain.step()
    host_in = host_out = None
    if h2d:
        host_in = torch.empty_like(chain.x_hidden, device="cpu").pin_memory()
        host_in.copy_(chain.x_hidden.cpu())
        host_out = torch.empty(out.shape, dtype=out.dtype, device="cpu").pin_memory()

    def one():
        with torch.cuda.stream(stream):
            if h2d:
                chain.x_hidden.copy_(host_in, non_blocking=True)
            graph.replay()
            if h2d:
                host_out.copy_(out, non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        one()
    t1.record(stream)
    torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / steps
    if world > 1:
        v = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        ms = float(v.item())
        dist.barrier()
    io = None
    if h2d:
        io = (host_in.numel() * host_in.element_size(), host_out.numel() * host_out.element_size())
    del graph
    return ms, io


def kernel_times(chain, device, reps=3):
    """Device time per launch of every fused decode + GEMV, per linear: one
    CUDA graph per linear name holding that linear's launch for every layer
    (distinct tensors, no L2 reuse, no host gaps), replayed `reps` times
    between events on the replay stream. The roofline's achieved bandwidth
    = algorithmic bytes (radix_ops.read_bytes + activations in and out) /
    device time."""
    import torch

    from drinkme_b200 import radix_ops

    stream = torch.cuda.Stream(device)
    out = {}
    tot_bytes = tot_ms = 0.0
    launches = 0
    for j, (name, parts) in enumerate(chain.groups):
        items = [(li, row[j]) for li, row in enumerate(chain.layers) if row[j] is not None]
        if not items:
            continue
        R, C = sum(p[1] for p in parts), parts[0][2]
        x = chain.inputs(j)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for li, rt in items:
                radix_ops.gemv_into(rt, x, None, chain.outs[li][j][:, :rt["R"]])
        g.replay()
        torch.cuda.synchronize(device)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            for _ in range(reps):
                g.replay()
            b.record(stream)
        torch.cuda.synchronize(device)
        ms = a.elapsed_time(b) / (reps * len(items))
        rt = items[0][1]
        nbytes = radix_ops.read_bytes(rt) + x.numel() * 2 + rt["R"] * 2
        us = ms * 1e3
        out[name] = {"shape": [R, C], "rows_here": rt["R"], "us": round(us, 2),
                     "compressed_gbs": round(nbytes / us * 1e-3, 1),
                     "bf16_equiv_gbs": round(rt["R"] * C * 2 / us * 1e-3, 1)}
        tot_bytes += nbytes * len(items)
        tot_ms += ms * len(items)
        launches += len(items)
        del g
    return out, tot_bytes, tot_ms, launches


def _graph_us(fn, device, reps=10):
    """Device µs of one replay of a CUDA graph of fn() (events on the replay
    stream, after a warm replay)."""
    import torch

    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    g.replay()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        a.record(s)
        for _ in range(reps):
            g.replay()
        b.record(s)
    torch.cuda.synchronize(device)
    us = a.elapsed_time(b) / reps * 1e3
    del g
    return us


def rotated_linear_us(profile, Ms, device):
    """µs per call of every Qwen3-8B linear on its own (one launch per linear,
    no fusion) for each activation row count in `Ms`: the shape's pack
    cloned into enough HBM copies to exceed 3x L2, one CUDA graph over the
    copies. Returns ({name: {M: us}}, {name: (read_bytes, device_bytes, bpw)})."""
    import torch

    from drinkme_b200 import codec, radix_ops, swap

    us, meta = {}, {}
    for j, (name, R, C) in enumerate(WORKLOADS["qwen3-8b"]["linears"]):
        bits = make_bits(R, C, seed=1000 + j, device=device)
        p = codec.pack_array_radix(bits, profile)
        rt0 = swap.to_device_radix(p, device)
        n = max(3, int(3 * 126e6 // radix_ops.read_bytes(rt0)) + 1)
        rts = [rt0] + [dict(rt0, rx_handle=rt0["rx_handle"].clone()) for _ in range(n - 1)]
        meta[name] = (radix_ops.read_bytes(rt0), int(rt0["rx_handle"].info.device_bytes_per_call), p["bpw"])
        for M in Ms:
            g = torch.Generator(device=device)
            x = torch.cat([torch.randn((1, C), generator=g.manual_seed(100 + m), device=device)
                           for m in range(M)]).to(torch.bfloat16)
            outs = [torch.empty((M, R), dtype=torch.bfloat16, device=device) for _ in rts]
            us.setdefault(name, {})[M] = _graph_us(
                lambda: [radix_ops.gemv_into(rt, x, None, o) for rt, o in zip(rts, outs)], device) / n
        del rts, outs, bits, p
        torch.cuda.empty_cache()
    return us, meta


def config3_gulp_mc(device, peak):
    """the Qwen3-8B linears packed gulp, through the
    narrow linear (radix_ops.gemv_mc_fused) with M = 2, 4, 8 rows (and M = 1
    beside them): µs per linear summed over one layer's seven linears, each
    shape rotated over copies larger than 3x L2, and the GB/s on the gulp
    read_bytes (the loader serves gulp through the sip kernels)."""
    Ms = (1, 2, 4, 8)
    us, meta = rotated_linear_us("gulp", Ms, device)
    total_bytes = sum(m[0] for m in meta.values())
    rows = {M: sum(us[n][M] for n in us) for M in Ms}
    res = {n: {**{f"M{M}_us": round(us[n][M], 2) for M in Ms}, "bpw": meta[n][2],
               "device_bytes_per_call": meta[n][1]} for n in us}
    summary = {f"M{M}": {"layer_us": round(t, 2), "gulp_gbs": round(total_bytes / t * 1e-3, 1),
                         "frac_of_peak": round(total_bytes / t * 1e-3 / peak, 4),
                         "us_per_row": round(t / M, 2)} for M, t in rows.items()}
    return {"config": "BASELINE configs[2]: Qwen3-8B linears packed gulp, M = 2/4/8 activation rows",
            "per_layer": summary, "per_linear": res,
            "note": "gulp packs with whole 1024-weight blocks are re-encoded as sip by the loader (same bits)"}


def vs_cublas_8b(device, peak):
    """north_star's M = 1 comparison on Qwen3-8B shapes: every linear (sip,
    one launch each) against cuBLAS dense bf16 (F.linear) on the uncompressed
    weight of the same shape, both rotated over copies larger than 3x L2.
    BF16-equivalent GB/s = R * C * 2 / time; ratio = cuBLAS µs / ours."""
    us, meta = rotated_linear_us("sip", (1,), device)
    cb = cublas_arm(WORKLOADS["qwen3-8b"]["linears"], device)
    out = {}
    for name, R, C in WORKLOADS["qwen3-8b"]["linears"]:
        ours = us[name][1]
        nbytes = meta[name][0] + C * 2 + R * 2
        out[name] = {"shape": [R, C], "ours_us": round(ours, 2), "cublas_us": cb[name]["us"],
                     "ratio_vs_cublas": round(cb[name]["us"] / ours, 3),
                     "ours_bf16_equiv_gbs": round(R * C * 2 / ours * 1e-3, 1),
                     "cublas_gbs": cb[name]["gbs"], "compressed_gbs": round(nbytes / ours * 1e-3, 1),
                     "frac_of_peak": round(nbytes / ours * 1e-3 / peak, 4)}
    t_ours = sum(v["ours_us"] for v in out.values())
    t_cb = sum(v["cublas_us"] for v in out.values())
    return {"config": "Qwen3-8B linears at M = 1, sip, one launch per linear, vs cuBLAS bf16 F.linear",
            "per_linear": out, "layer_ratio_vs_cublas": round(t_cb / t_ours, 3)}


def config5_prefill(device):
    """x [512, C] against sip gate/up 12288x4096 and down
    4096x12288: the package's prefill route (CompressedLinear's dense arm: the
    sip pipeline's decode mode to bf16, then cuBLAS) next to cuBLAS bf16 on
    the uncompressed weights; TFLOP/s = 2 * 512 * R * C / time."""
    import torch

    from drinkme_b200 import codec, radix_ops, swap

    out = {}
    for name, R, C in (("gate", 12288, 4096), ("up", 12288, 4096), ("down", 4096, 12288)):
        bits = make_bits(R, C, seed=7 + R + C, device=device)
        p = codec.pack_array_radix(bits, "sip")
        rt = swap.to_device_radix(p, device)
        x = torch.randn((512, C), generator=torch.Generator(device=device).manual_seed(2),
                        device=device).to(torch.bfloat16)
        ws = [(torch.randn((R, C), device=device) * 0.02).to(torch.bfloat16) for _ in range(3)]
        us_cublas = _graph_us(lambda: [torch.nn.functional.linear(x, w) for w in ws], device) / 3
        us_decode = _graph_us(lambda: radix_ops.decode_weight(rt), device)
        us_path = _graph_us(lambda: torch.nn.functional.linear(x, radix_ops.decode_weight(rt)), device)
        us_tc = _graph_us(lambda: radix_ops.prefill(rt, x, None, torch.bfloat16), device)
        fl = 2 * 512 * R * C
        out[name] = {"path_us": round(us_path, 2), "path_tflops": round(fl / us_path * 1e-6, 1),
                     "decode_us": round(us_decode, 2), "cublas_bf16_us": round(us_cublas, 2),
                     "cublas_tflops": round(fl / us_cublas * 1e-6, 1),
                     "tcgen05_prefill_us": round(us_tc, 2), "tcgen05_prefill_tflops": round(fl / us_tc * 1e-6, 1)}
        del ws, rt, p, bits
        torch.cuda.empty_cache()
    return {"config": "BASELINE configs[4]: prefill x [512, C], sip gate/up/down of Qwen3-8B",
            "route": "decode to bf16 (sip pipeline, decode mode) then cuBLAS; tcgen05_* = the fused tensor-core "
                     "prefill kernel (decoded tiles in shared memory, TMEM accumulators)", "per_linear": out}


def crossover_8b(device, Ms=(8, 9, 12, 16, 24, 32, 48, 64)):
    """The row count at which the dense arm starts to beat the multi-column
    GEMV on B200 (the measurement DRINKME_PREFILL_DENSE_MIN exists for,
    swap.py:205-225): one Qwen3-8B layer's seven sip linears at M activation
    rows through (a) the row loop in chunks of MC_MAX rows on the mc kernel,
    (b) the reference's dense arm, decode to bf16 then cuBLAS, (c) the
    tensor-core prefill kernel; µs per layer from one CUDA graph per arm."""
    import torch

    from drinkme_b200 import codec, radix_ops, swap
    from drinkme_b200.ops import MC_MAX

    lins = []
    for j, (name, R, C) in enumerate(WORKLOADS["qwen3-8b"]["linears"]):
        bits = make_bits(R, C, seed=3000 + j, device=device)
        lins.append((name, swap.to_device_radix(codec.pack_array_radix(bits, "sip"), device), R, C))
        del bits
    rows = {}
    for M in Ms:
        xs = {C: (torch.randn((M, C), generator=torch.Generator(device=device).manual_seed(M), device=device)
                  .to(torch.bfloat16)) for C in {c for _, _, _, c in lins}}
        outs = [torch.empty((M, R), dtype=torch.bfloat16, device=device) for _, _, R, _ in lins]

        def loop():
            for (_, rt, R, C), o in zip(lins, outs):
                for i in range(0, M, MC_MAX):
                    radix_ops.gemv_into(rt, xs[C][i:i + MC_MAX], None, o[i:i + MC_MAX])

        def dense():
            for (_, rt, R, C), o in zip(lins, outs):
                o.copy_(torch.nn.functional.linear(xs[C], radix_ops.decode_weight(rt)))

        def tc():
            for (_, rt, R, C), o in zip(lins, outs):
                o.copy_(radix_ops.prefill(rt, xs[C], None, torch.bfloat16))

        rows[M] = {"mc_loop_us": round(_graph_us(loop, device), 1), "dense_us": round(_graph_us(dense, device), 1),
                   "tcgen05_us": round(_graph_us(tc, device), 1)}
        del xs, outs
    dense_min = next((M for M in Ms if rows[M]["dense_us"] < rows[M]["mc_loop_us"]), None)
    del lins
    torch.cuda.empty_cache()
    return {"config": "Qwen3-8B layer (7 sip linears) at M activation rows: mc in chunks of MC_MAX vs decode + cuBLAS "
                      "vs the tcgen05 prefill kernel, us per layer", "per_M": rows,
            "dense_beats_mc_from_M": dense_min}


def decode_step_8b(device, steps=20, warmup=3):
    """SURVEY (f) 3: a whole batch-1 Qwen3-8B decode step (36 layers: norms,
    q|k|v, rotary, KV-cache attention, o, gate|up, SiLU, down, lm_head,
    greedy sampling) replayed from one CUDA graph (decode_step.DecodeStack),
    tokens/s from device-timed replays at positions 0..steps."""
    import torch

    from drinkme_b200 import decode_step

    st = decode_step.DecodeStack(decode_step.QWEN3["qwen3-8b"], device, max_len=1024, seed=11)
    st.reset(token=1)
    st.capture()
    for _ in range(warmup):
        st.replay()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        st.replay()
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b) / steps
    # the same graph at a long context: positions 896.. (the rows below are
    # whatever the cache holds; only the timing is read)
    st.pos.fill_(896)
    for _ in range(warmup):
        st.replay()
    torch.cuda.synchronize(device)
    a.record()
    for _ in range(steps):
        st.replay()
    b.record()
    torch.cuda.synchronize(device)
    ms_long = a.elapsed_time(b) / steps
    out = {"config": "Qwen3-8B shapes, 36 layers, sip linears + raw bf16 lm_head, batch 1, KV cache of 1024 rows "
                     "(attention over the allocation with a live-length mask), one CUDA graph per step",
           "ms_per_step": round(ms, 4), "tokens_per_s": round(1e3 / ms, 2), "steps": steps,
           "positions": f"0..{warmup + steps - 1}", "ms_per_step_at_position_896": round(ms_long, 4),
           "graph_nodes_note": "per layer: the sip linears (q|k|v, o, gate|up, down), residual add + RMSNorm twice, the "
                               "attention block (q/k norm, rotary, cache write, split attention and combine in one "
                               "launch) and SiLU * up are this package's kernels; the embedding lookup, greedy argmax "
                               "and position counter are torch operations"}
    del st
    torch.cuda.empty_cache()
    return out


def cublas_arm(shapes, device, reps=10):
    """cuBLAS dense bf16 (F.linear, M = 1) on uncompressed weights of the same
    shapes, rotating over copies larger than 3x L2 inside one CUDA graph (as
    this package's launches are timed): µs per call and GB/s."""
    import torch

    res = {}
    for name, R, C in shapes:
        copies = max(2, int(3 * 126e6 // (R * C * 2)) + 1)
        ws = [(torch.randn((R, C), device=device) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn((1, C), device=device).to(torch.bfloat16)
        us = _graph_us(lambda: [torch.nn.functional.linear(x, w) for w in ws], device, reps) / copies
        res[name] = {"shape": [R, C], "us": round(us, 2), "gbs": round(R * C * 2 / us * 1e-3, 1)}
        del ws
        torch.cuda.empty_cache()
    return res


# --------------------------------------------------------- CPU reference --

def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_reference(wl, steps, warmup, log=lambda m: None):
    """The reference's CPU route on the host (swap.CompressedLinear "cpu",
    swap.py:344-352): every linear decoded once by the reference's own native
    decoder (radix_pack.decode_back_radix -> radix_native.decode, compiled
    from its sources into oracle/_ref), then torch F.linear over the cached
    bf16 weight on every call. Weights are packed by the reference's own
    native encoder (radix_native plan + encode), never by this package, whose
    library this arm does not load.

    A step is one token of the named stack: the 7 linears of one layer,
    decoded once, run layers (64) times, i.e. the whole stack's F.linear work;
    the one layer's weights (about 1 GB for Qwen3-32B) are far larger than
    the host's last-level cache, so every pass streams them from DRAM as
    distinct layers would. `warmup` untimed steps, then `steps` timed ones,
    every host thread. Returns (tokens/s, fields)."""
    import numpy as np
    import torch

    from oracle import oracle

    spec = WORKLOADS[wl]
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)  # every host thread, also under torchrun
    if oracle.reference_native() is None:
        raise RuntimeError("the reference's native codec is not built (make -C oracle REF_SRC=...)")
    g = torch.Generator().manual_seed(7)
    ws, xs, packs = [], {}, []
    t_pack = t_dec = 0.0
    for name, R, C in spec["linears"]:
        w = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        bits = w.view(torch.int16).numpy().view(np.uint16)
        t0 = time.perf_counter()
        p = oracle.reference_encode(bits, (3, 8))
        t1 = time.perf_counter()
        dec = oracle.reference_decode(p)  # single-threaded, the route's first call
        t_dec += time.perf_counter() - t1
        t_pack += t1 - t0
        assert np.array_equal(dec, bits), f"{name}: the reference's decode differs from the source bits"
        ws.append(torch.from_numpy(dec.view(np.int16)).view(torch.bfloat16))
        packs.append(p)
        if C not in xs:
            xs[C] = torch.randn(1, C, generator=g).to(torch.bfloat16)
        del w
    log(f"reference CPU: packed one layer in {t_pack:.1f}s, decoded in {t_dec:.1f}s")
    nweights = sum(int(w.numel()) for w in ws)
    # decode throughput, one thread and every thread (radix_native.decode workers=1 / N)
    big = max(range(len(packs)), key=lambda i: ws[i].numel())
    t0 = time.perf_counter()
    oracle.reference_decode_threads(packs[big], 1)
    d1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    oracle.reference_decode_threads(packs[big], cores)
    dn = time.perf_counter() - t0
    # cold call of the largest linear: decode + the first F.linear
    t0 = time.perf_counter()
    wc = torch.from_numpy(oracle.reference_decode(packs[big]).view(np.int16)).view(torch.bfloat16)
    torch.nn.functional.linear(xs[wc.shape[1]], wc)
    cold = time.perf_counter() - t0
    del packs, wc

    def step():
        for _ in range(spec["layers"]):
            for w in ws:
                torch.nn.functional.linear(xs[w.shape[1]], w)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    secs = time.perf_counter() - t0
    tok_s = steps / secs
    fields = {
        "cores": torch.get_num_threads(), "os_cpu_count": cores, "cpu_model": cpu_model(),
        "cold_call_s": round(cold, 4),
        "decode_weights_per_s_workers1": round(ws[big].numel() / d1, 1),
        "decode_weights_per_s_workersN": round(ws[big].numel() / dn, 1), "decode_workers_N": cores,
        "sample": (f"one token of the {spec['layers']}-layer stack per step: one layer's {len(ws)} linears "
                   f"({nweights / 1e6:.0f}M weights, packed and decoded by the reference's own native codec) "
                   f"run {spec['layers']} times through torch F.linear on {torch.get_num_threads()} threads "
                   f"({warmup} warm-up + {steps} timed steps; the layer's bf16 weights stream from DRAM every "
                   f"pass)"),
    }
    return tok_s, fields


# ------------------------------------------------------------------ main --

def main():
    a = parse()
    world, rank, local = dist_env()
    if a.gpus != world and world > 1:
        print(f"warning: --gpus {a.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if a.layers:
        for wl in WORKLOADS.values():
            wl["layers"] = a.layers
    spec = WORKLOADS[a.workload]
    base_config = {"workload": f"{a.workload} decode linear stack, batch 1, sip, row-sharded over {world} GPU(s)"
                               + ("" if a.no_fuse else "; q|k|v and gate|up fused launches")
                               + ("" if world == 1 else f"; output gather: {a.gather}"),
                   "model_shape": a.workload, "layers": spec["layers"], "global_batch": 1,
                   "parallelism": f"rows{world}", "l2": "inputs larger than L2 (stack >> 126 MB)"}

    if a.impl == "reference":
        if rank != 0:
            return 0
        log = (lambda m: print(f"[bench] {m}", file=sys.stderr, flush=True))
        tok_s, f = cpu_reference(a.workload, a.steps, a.warmup, log)
        line = {"metric": METRIC, "value": round(tok_s, 4), "unit": "tokens/s",
                "impl": "reference", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": round(1e3 / tok_s, 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic: N(0,0.02) bf16 weights packed sip by the reference's native encoder, "
                        "N(0,1) bf16 activations",
                "config": base_config,
                "cpu_baseline": {"value": round(tok_s, 4), "unit": "tokens/s", "kind": "reference", **f},
                "e2e": {"value": round(tok_s, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))

    def log(msg):
        if rank == 0:
            print(f"[bench] {msg}", file=sys.stderr, flush=True)

    fuse = not a.no_fuse
    layers, stats = build_stack(a.workload, rank, world, device, a.variants, log, fuse)
    if a.launch == "auto":
        a.launch = "linear"
    chain = Chain(a.workload, layers, rank, world, device, fuse=fuse, gather=a.gather, launch=a.launch)
    clocks = ClockSampler(local)
    clocks.start()
    ms, _ = time_graph(chain, a.steps, a.warmup, world, rank, device)
    clk = clocks.stop()
    ms_e2e, io = time_graph(chain, a.steps, max(3, a.warmup), world, rank, device, h2d=True)
    per_kernel, tot_bytes, tot_ms, launches = kernel_times(chain, device)
    # the same step in the other launch mode
    other = "linear" if a.launch == "chain" else ("chain" if world == 1 or a.gather == "peer" else None)
    ms_other = None
    if other is not None:
        alt = Chain(a.workload, layers, rank, world, device, fuse=fuse, gather=a.gather, launch=other)
        ms_other, _ = time_graph(alt, a.steps, a.warmup, world, rank, device)
        alt.close()
        del alt
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    # the dominant kernel: the chain launch (the whole step) or the
    # per-linear launches (their device time summed)
    k_ms = ms if a.launch == "chain" else tot_ms
    achieved = tot_bytes / (k_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if os.path.exists(tpath):
        with open(tpath) as f:
            for line in f:
                if line.startswith(f"{a.workload}_bytes_per_launch:"):
                    traffic = float(line.split(":", 1)[1])
    words = sum(v["words"] for v in stats.values())
    result = None
    if rank == 0:
        tok_s = 1e3 / ms
        result = {
            "metric": METRIC,
            "value": round(tok_s, 3), "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: N(0,0.02) bf16 weights packed sip (byte-identical encoder), "
                                     "N(0,1) bf16 activations",
            "config": base_config,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "sip_chain_kernel" if a.launch == "chain" else "sip_gemv_kernel",
                         "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)",
                         "bytes_per_step_algorithmic": int(tot_bytes), "kernel_ms_per_step": round(k_ms, 4)},
            "launch": ("one persistent launch per step over every linear (dm_chain_run; link k waits for link "
                       "k - 1's flags)" if a.launch == "chain" else "one launch per linear (dm_gemv / "
                       "dm_gemv_gather)"),
            "per_linear": per_kernel,
            "e2e": {"value": round(1e3 / ms_e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": io[0],
                    "d2h_bytes_per_step": io[1]},
            "gpu_launches": chain.launches_per_step() * a.steps,
            "other_launch": None if ms_other is None else {
                "launch": other, "tokens_per_s": round(1e3 / ms_other, 3), "ms_per_step": round(ms_other, 4),
                "note": "the same step and bits in the other launch mode (chain: one sip_chain_kernel launch; "
                        "linear: one sip_gemv_kernel launch per linear)"},
            "clocks": clk,
            "pack": {"variants_per_shape": a.variants, "bpw_mean": round(
                sum(v["bpw"] for v in stats.values()) / len(stats), 4), "distinct_words": words},
        }
    if world == 1 and rank == 0:
        if not a.no_cublas:
            result["cublas_dense_bf16"] = cublas_arm([(n, R, C) for n, R, C in spec["linears"] if n != "v"], device)
        if not a.no_secondary and a.workload != "qwen3-8b":
            del chain, layers
            torch.cuda.empty_cache()
            l8, _ = build_stack("qwen3-8b", 0, 1, device, a.variants, log, fuse)
            g = torch.Generator(device=device).manual_seed(3)
            head = (torch.randn(WORKLOADS["qwen3-8b"]["head"], generator=g, device=device) * 0.02).to(torch.bfloat16)
            c8 = Chain("qwen3-8b", l8, 0, 1, device, head_weight=head, fuse=fuse, launch=a.launch)
            ms8, _ = time_graph(c8, a.steps, a.warmup, 1, 0, device)
            c8o = Chain("qwen3-8b", l8, 0, 1, device, head_weight=head, fuse=fuse, launch=other)
            ms8_other, _ = time_graph(c8o, a.steps, a.warmup, 1, 0, device)
            c8o.close()
            del c8o
            pk8, b8, t8, _ = kernel_times(c8, device)
            # the raw bf16 lm_head alone: this package's raw GEMV and cuBLAS
            from drinkme_b200 import radix_ops
            xh = torch.randn((1, head.shape[1]), generator=g, device=device).to(torch.bfloat16)
            hb = head.numel() * 2 + xh.numel() * 2 + head.shape[0] * 2
            h_us = _graph_us(lambda: radix_ops.gemv_raw(head, xh, None, torch.bfloat16), device)
            h_cublas = _graph_us(lambda: torch.nn.functional.linear(xh, head), device)
            result["qwen3_8b_chain"] = {"config": "BASELINE configs[1]: 36 layers + raw lm_head 151936x4096",
                                        "tokens_per_s": round(1e3 / ms8, 3), "ms_per_step": round(ms8, 4),
                                        "launch": a.launch,
                                        "other_launch": {"launch": other,
                                                         "tokens_per_s": round(1e3 / ms8_other, 3)},
                                        "fused_gemv_gbs": round(b8 / (t8 * 1e-3) / 1e9, 1),
                                        "frac_of_peak": round(b8 / (t8 * 1e-3) / 1e9 / peak, 4),
                                        "per_linear": pk8,
                                        "lm_head_raw": {"us": round(h_us, 2), "gbs": round(hb / h_us * 1e-3, 1),
                                                        "frac_of_peak": round(hb / h_us * 1e-3 / peak, 4),
                                                        "cublas_us": round(h_cublas, 2)}}
        if not a.no_configs:
            result["vs_cublas_8b_m1"] = vs_cublas_8b(device, peak)
            result["config3_gulp_mc"] = config3_gulp_mc(device, peak)
            result["config5_prefill"] = config5_prefill(device)
            result["crossover_8b"] = crossover_8b(device)
            result["decode_step_8b"] = decode_step_8b(device)
        if not a.no_cpu:
            tok_s, f = cpu_reference(a.workload, 3, 1, log)
            result["cpu_baseline"] = {"value": round(tok_s, 4), "unit": "tokens/s", "kind": "reference", **f}
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist

        chain.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
