"""bench.py -- PPO train samples/s of the PTCG policy hot path on B200.

Headline (BASELINE.json metric, config 2 / 3): one PPO minibatch step =
forward (all heads) + fused clipped-PPO/value/entropy loss + backward +
global-norm clip + fused Adam, 512 segments x 64 steps = 32768 samples per
GPU of config-0-shaped observations (d256, 4 layers, 8 heads, FFN 1024,
128 tokens, 64 options), bf16 tensor-core GEMMs with fp32 accumulation.
Data parallel over N GPUs (torchrun, one process per GPU): every rank trains
on its own minibatch (seed + rank); gradient buckets are all-reduced over
NCCL on a side stream as the backward produces them, then every rank runs
the same Adam; weights are checked identical across ranks each step.

Also reported: rollout forward/s (config 1: 1024 agents x 64 env steps,
forward + masked sampling), end-to-end numbers through the public API with
host<->device copies, the roofline of the dominant kernel, and the CPU
baseline (the CPU oracle on the host cores).

--impl reference times the reference's own CPU implementation on the host
cores: its torch model (ptcg/rl/model.py PTCGTransformer, from the offline
install under baseline/_ref) with the PPO loss gradients of its kernel,
autograd and torch Adam.  Where that install is absent, the CPU oracle port
stands in and the line says kind "port".
"""
import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--preset", default="c0")
    ap.add_argument("--segments", type=int, default=None,
                    help="train segments per GPU (config 2: 512; config 4: 1024)")
    ap.add_argument("--horizon", type=int, default=64)
    ap.add_argument("--micro", type=int, default=None,
                    help="rows per micro-batch (c0: 16384; c4: 1024)")
    ap.add_argument("--rollout-agents", type=int, default=None,
                    help="rollout agents per GPU (config 1: 1024; config 4: 4096)")
    ap.add_argument("--dp", default="sharded", choices=["allreduce", "sharded", "native"],
                    help="N>1 gradient exchange: bucketed all-reduce + Adam on every rank; "
                         "bucketed reduce-scatter + Adam on each rank's shard + all-gather "
                         "driven from Python (sharded); or the same exchange issued by the "
                         "library itself over NCCL (native)")
    ap.add_argument("--rollout-graph", type=int, default=1,
                    help="replay the rollout forward + sampler as a CUDA graph")
    ap.add_argument("--rollout-steps", type=int, default=64)
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-rollout", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ref-rows", type=int, default=128,
                    help="observations per step of the reference (CPU) arm")
    a = ap.parse_args()
    # c0 shapes for configs 0-3, the scaled policy for 4
    d = PRESET_DEFAULTS.get(a.preset, PRESET_DEFAULTS["c0"])
    a.segments = a.segments or d["segments"]
    a.micro = a.micro or d["micro"]
    a.rollout_agents = a.rollout_agents or d["rollout_agents"]
    return a


PRESET_DEFAULTS = {
    "c0": {"segments": 512, "micro": 16384, "rollout_agents": 1024},
    "c4": {"segments": 1024, "micro": 1024, "rollout_agents": 4096},
}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- reference
METRICS = {"c0": "PPO train samples/sec (config 2 per GPU, aggregate)",
           "c4": "PPO train samples/sec (config 4 per GPU, aggregate)"}


def metric_name(preset):
    return METRICS.get(preset, f"PPO train samples/sec ({preset} per GPU, aggregate)")
REF_INSTALL = os.path.join(ROOT, "baseline", "_ref")


def reference_installed():
    """The reference's torch model is importable from baseline/_ref."""
    return os.path.exists(os.path.join(REF_INSTALL, "ptcg", "rl", "model.py"))


def _ref_model(pkg, s):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref_torch
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    return ref_torch, ref_torch.load(REF_INSTALL, s, tabs, blob, pkg.config.param_table)


def cpu_reference_step(pkg, s, rows, threads):
    """One train step of the reference's own torch model (forward_train, PPO
    loss gradients, aux losses, backward, clip, torch Adam) on `rows`
    config-shaped observations, as a callable."""
    import torch
    torch.set_num_threads(threads)
    ref_torch, model = _ref_model(pkg, s)
    obs = pkg.synth.make_obs_batch(s, rows, 5)
    a, b = s.offsets["opt_mask"]
    act = pkg.synth.sample_legal(obs[:, a:b], 1)
    rng = np.random.default_rng(0)
    adv = rng.standard_normal(rows).astype(np.float32)
    ret = rng.standard_normal(rows).astype(np.float32)
    old = np.full(rows, -2.0, np.float32)
    val = np.zeros(rows, np.float32)
    return ref_torch.train_step(model, s, obs, act, old, adv, val, ret, np.ones(1, np.float32),
                                1, rows)


def cpu_step(pkg, s, rows, threads):
    """(step callable, kind): the reference's torch model when installed,
    else the CPU oracle port."""
    if reference_installed():
        return cpu_reference_step(pkg, s, rows, threads), "reference"
    return cpu_oracle_step(pkg, s, rows, threads), "port"


def arm_config(args, s, world, micro):
    nt = args.segments * args.horizon
    return {"workload": f"ppo_train_step {args.preset}: {args.segments}x{args.horizon} "
                        f"samples/GPU, micro-batch {micro}",
            "model": "PTCGTransformer d%d L%d h%d ffn%d ltok%d nopt%d" % (
                s.d, s.layers, s.heads, s.ffn, s.ltok, s.nopt),
            "global_batch": nt * world, "seq_len": s.lseq,
            "parallelism": f"dp{world}" + ("" if world == 1 else f" ({args.dp})"),
            "l2": "inputs larger than L2 (obs %.0f MB per step per GPU)" % (
                nt * s.obs_size * 4 / 1e6)}


def cpu_oracle_step(pkg, s, rows, threads):
    """One CPU oracle train step (forward_train + PPO loss + backward + clip +
    Adam) on `rows` config-shaped observations, as a callable."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ptcg_oracle as oracle
    torch.set_num_threads(threads)
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    obs = pkg.synth.make_obs_batch(s, rows, 5)
    a, b = s.offsets["opt_mask"]
    act = pkg.synth.sample_legal(obs[:, a:b], 1)
    rng = np.random.default_rng(0)
    P = oracle.params_from_blob(blob, s, requires_grad=True)
    T = oracle.tables_to_torch(tabs)
    state = {}
    adv = rng.standard_normal(rows).astype(np.float32)
    ret = rng.standard_normal(rows).astype(np.float32)
    old = np.full(rows, -2.0, np.float32)
    val = np.zeros(rows, np.float32)
    prio = np.ones(1, np.float32)

    def step():
        _, _, g = oracle.train_grads(P, T, obs, s, act, old, adv, val, ret, prio, 1, rows)
        oracle.adam_step(P, g, state)
    return step


def cpu_step_rate(pkg, s, rows, seconds, threads, port_only=False):
    """Samples/s of a CPU train step (cpu_step), median over ~`seconds`."""
    if port_only:
        step, kind = cpu_oracle_step(pkg, s, rows, threads), "port"
    else:
        step, kind = cpu_step(pkg, s, rows, threads)
    step()                                  # warm-up
    times = []
    t_end = time.time() + seconds
    while time.time() < t_end or len(times) < 2:
        t0 = time.time(); step(); times.append(time.time() - t0)
    med = float(np.median(times))
    return rows / med, len(times), med, kind


def cpu_rollout_rate(pkg, s, rows, seconds, threads):
    """Observations/s of a CPU rollout forward (forward_eval under no_grad)
    on `rows` config-shaped observations, median over ~`seconds`: the
    reference's torch model when installed, else the CPU oracle port."""
    import torch
    torch.set_num_threads(threads)
    obs = torch.from_numpy(pkg.synth.make_obs_batch(s, rows, 6))
    if reference_installed():
        _, model = _ref_model(pkg, s)
        fwd, kind = (lambda: model.forward_eval(obs)), "reference"
    else:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import ptcg_oracle as oracle
        P = oracle.params_from_blob(pkg.synth.make_weights(s, 21), s)
        T = oracle.tables_to_torch(pkg.synth.make_tables(s, 11))
        fwd, kind = (lambda: oracle.forward_eval(P, T, obs, s)), "port"
    times = []
    with torch.no_grad():
        fwd()                                         # warm-up
        t_end = time.time() + seconds
        while time.time() < t_end or len(times) < 2:
            t0 = time.time(); fwd(); times.append(time.time() - t0)
    med = float(np.median(times))
    return rows / med, len(times), med, kind


def run_reference(args, pkg):
    """The reference arm: the reference's own CPU implementation (its torch
    PTCGTransformer, PPO loss gradients, autograd, torch Adam; the oracle
    port where baseline/_ref is absent) on all host cores; each step is a
    bounded sample of the config-2 workload (--ref-rows observations of the
    same shapes); W warm-up then K timed steps."""
    s = pkg.config.PRESETS[args.preset]
    threads = os.cpu_count() or 1
    rows = args.ref_rows
    step, kind = cpu_step(pkg, s, rows, threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    rate = rows * args.steps / dt
    what = ("the reference's torch PTCGTransformer (baseline/_ref)" if kind == "reference"
            else "the CPU oracle port")
    sample = (f"{rows}-row PPO train step of {what} (forward_train + PPO loss + aux losses + "
              f"backward + clip + Adam) per step, {threads} threads")
    nt = args.segments * args.horizon
    cfg = arm_config(args, s, args.gpus, min(args.micro, nt))
    cfg["sample_rows_per_step"] = rows
    line = {"impl": "reference", "metric": metric_name(args.preset),
            "value": rate, "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": rate, "unit": "samples/s", "cores": threads,
                             "kind": kind, "sample": sample},
            "e2e": {"value": rate, "unit": "samples/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- ours
def main():
    args = parse()
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, pkg)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    s = pkg.config.PRESETS[args.preset]
    nt = args.segments * args.horizon
    micro = min(args.micro, nt)
    tabs = pkg.synth.make_tables(s, 11)
    blob = pkg.synth.make_weights(s, 21)
    pol = pkg.PTCGPolicy(s, precision="bf16", device=local, tables=tabs, weights=blob,
                         rollout_rows=args.rollout_agents, train_rows=micro)

    # --- this rank's minibatch (config 2/3): pool of distinct rows, tiled
    pool_n = min(nt, 8192)
    pool = pkg.synth.make_obs_batch(s, pool_n, 1000 + rank)
    reps = (nt + pool_n - 1) // pool_n
    order = np.random.default_rng(7 + rank).permutation(reps * pool_n)[:nt] % pool_n
    obs_h = torch.from_numpy(pool[order]).pin_memory()
    a, b = s.offsets["opt_mask"]
    act_h = torch.from_numpy(pkg.synth.sample_legal(obs_h[:, a:b].numpy(), 3 + rank))
    obs = obs_h.to(dev)
    act = act_h.to(dev)
    # old log-probs and values from the forward pass (rollout path)
    old = torch.empty(nt, device=dev)
    vals = torch.empty(nt, device=dev)
    for c0 in range(0, nt, args.rollout_agents):
        c1 = min(nt, c0 + args.rollout_agents)
        out = pol.forward(obs[c0:c1])
        m = obs[c0:c1, a:b]
        lg = out[:, :-1].masked_fill(m == 0, -1e4)
        lp = torch.log_softmax(lg, 1)
        old[c0:c1] = lp.gather(1, act[c0:c1].long()[:, None])[:, 0]
        vals[c0:c1] = out[:, -1]
    g = torch.Generator(device="cpu").manual_seed(99 + rank)
    adv = torch.randn(nt, generator=g).to(dev)
    ret = torch.randn(nt, generator=g).to(dev)
    prio = torch.ones(args.segments, device=dev)
    hyper = dict(clip=0.2, vf_clip=0.2, vf_coef=0.5, ent_coef=0.01, lr=3e-4,
                 betas=(0.9, 0.999), eps=1e-8, max_norm=1.0)

    # --- data parallel: bucketed all-reduce overlapped with the backward
    grads = pol.arena(1)
    reducer = None
    native_dp = world > 1 and args.dp == "native"
    if native_dp:
        pol.dp_init()
    elif world > 1:
        from ptcg_b200.dp import BucketAllReduce, checksum_u64, weights_agree
        if args.dp == "sharded":
            reducer = pol.sharded_adam(lr=3e-4, betas=(0.9, 0.999), eps=1e-8, max_norm=1.0)
        else:
            reducer = BucketAllReduce(grads)
            pol.set_grad_hook(reducer)
    ck = torch.zeros(max(1, args.steps + args.warmup), 2, dtype=torch.int64, device=dev)
    stats = torch.zeros(16, device=dev)

    covered = []

    def step(i, o=obs, ac=act, ol=old, ad=adv, va=vals, re=ret):
        if reducer is not None:
            reducer.reset()
        pol.train_step(o, ac, ol, ad, va, re, prio, args.segments, args.horizon,
                       skip_adam=world > 1 and not native_dp, stats=stats, **hyper)
        if native_dp:
            pol.dp_weights_agree(ck[i])
        if reducer is not None:
            covered.append(reducer.covered(grads.numel()))
            if args.dp == "sharded":
                reducer.step(stats[8:10])       # {grad norm, applied} as train_step writes them
            else:
                reducer.wait()
                st2 = pol.adam_step(lr=hyper["lr"], betas=hyper["betas"], eps=hyper["eps"],
                                    max_norm=hyper["max_norm"])
                stats[8:10].copy_(st2)
            mn, mx = weights_agree(checksum_u64(pol.weights_checksum()))
            ck[i, 0] = mn; ck[i, 1] = mx

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    use_tc = pol.lib.ptcg_launch_count  # noqa: F841 (symbol presence)
    timer_mode = 1 if _tc_available(pol) else 2
    pol.kernel_timer(timer_mode)
    l0 = pol.lib.ptcg_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches = pol.lib.ptcg_launch_count() - l0
    kms, klaunch, kflops = pol.kernel_timer_read()
    kbytes = pol.kernel_timer_bytes()
    pol.kernel_timer(0)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        lt = torch.tensor([launches], device=dev, dtype=torch.int64)
        dist.all_reduce(lt)
        launches = int(lt.item())
        ok = bool((ck[:, 0] == ck[:, 1]).all().item())
    else:
        ok = True
    ms_max = float(t.item())
    ms_step = ms_max / args.steps
    value = nt * world * args.steps / (ms_max / 1e3)
    st = stats.cpu().numpy()

    # --- end to end through the public API: every step copies its inputs
    #     from pinned host memory (HostFeed: on a copy stream, the next
    #     step's inputs crossing PCIe while this step computes), runs the
    #     train step and reads the loss stats back to the host
    from ptcg_b200.feed import HostFeed
    host = dict(obs=obs_h, act=act_h.pin_memory(), old=old.cpu().pin_memory(),
                adv=adv.cpu().pin_memory(), val=vals.cpu().pin_memory(),
                ret=ret.cpu().pin_memory())
    feed = HostFeed(host, dev, depth=2)
    h2d = feed.bytes_per_put
    d2h = 16 * 4
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    feed.start()
    feed.put(host)
    for i in range(args.e2e_steps):
        fb = feed.get()
        if i + 1 < args.e2e_steps:
            feed.put(host)
        step(0, fb["obs"], fb["act"], fb["old"], fb["adv"], fb["val"], fb["ret"])
        feed.release()
        _ = stats.cpu()
    f1.record()
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = nt * world * args.e2e_steps / (float(te.item()) / 1e3)

    # the library's own exchange is done: the timings below are per GPU
    if native_dp:
        pol.dp_finalize()

    # --- optimizer roofline (HBM): ptcg_adam_step = norm pass + fused
    #     clip/Adam/bf16-copy pass, timed alone with CUDA events
    from ptcg_b200.config import optimizer_bytes
    ob = optimizer_bytes(s)["total"]
    import ctypes
    ost = torch.zeros(2, device=dev)
    cstream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def adam_call():
        pol.lib.ptcg_adam_step(pol.h, hyper["lr"], hyper["betas"][0], hyper["betas"][1],
                               hyper["eps"], hyper["max_norm"], None,
                               ctypes.c_void_p(ost.data_ptr()), cstream)
    for _ in range(3):
        adam_call()
    torch.cuda.synchronize()
    # the optimizer kernels alone (the library's CUDA events around the norm
    # and fused Adam launches); each step also refreshes the static-table
    # activations for the new weights, which is forward work, not optimizer
    pol.kernel_timer(4)
    for _ in range(20):
        adam_call()
    torch.cuda.synchronize()
    adam_kms, adam_n, _ = pol.kernel_timer_read()
    pol.kernel_timer(0)
    adam_ms = adam_kms / max(1, adam_n)

    # --- write-only HBM bandwidth of this GPU (a 2 GiB fp32 fill): the roof
    #     of GEMMs whose traffic is mostly their outputs.  torch's 1- and
    #     2-byte fills reach about half the rate of its 4-byte fill here, so
    #     the buffer is fp32
    wbuf = torch.empty(1 << 29, dtype=torch.float32, device=dev)
    for _ in range(3):
        wbuf.fill_(1.0)
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    w0.record()
    for _ in range(10):
        wbuf.fill_(2.0)
    w1.record()
    torch.cuda.synchronize()
    write_gbs = 10 * wbuf.numel() * wbuf.element_size() / (w0.elapsed_time(w1) / 1e3) / 1e9
    del wbuf

    # --- rollout forward (config 1): fresh observations every env step.
    #     With --rollout-graph the forward + sampler are one CUDA graph
    #     replayed per env step (the reference replays its rollout graph,
    #     pufferlib.cu:771-780); each step's observations and uniforms are
    #     copied into the graph's input buffers first, inside the timed loop.
    rollout = None
    graph = None
    if not args.no_rollout:
        A = args.rollout_agents
        nroll = 8
        ro_h = torch.from_numpy(pkg.synth.make_obs_batch(s, A * nroll, 500 + rank)).pin_memory()
        ro = ro_h.to(dev)
        uni = torch.rand(args.rollout_steps, A, device=dev)
        gsrc = torch.empty(A, s.obs_size, device=dev)
        guni = torch.empty(A, device=dev)

        def rstep_static():
            # forward with the sampler fused into its output kernel
            _, act_, lp_, v_ = pol.forward_sample(gsrc, guni)
            return act_, lp_, v_

        gsrc.copy_(ro[:A])
        guni.copy_(uni[0])
        if args.rollout_graph:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    rstep_static()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                gout = rstep_static()

        def rstep(j, src):
            gsrc.copy_(src, non_blocking=True)
            guni.copy_(uni[j])
            if graph is not None:
                graph.replay()
                return gout
            return rstep_static()

        for j in range(3):
            rstep(j, ro[:A])
        torch.cuda.synchronize()
        l0r = pol.lib.ptcg_launch_count()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for j in range(args.rollout_steps):
            k = j % nroll
            rstep(j, ro[k * A:(k + 1) * A])
        r1.record()
        torch.cuda.synchronize()
        rms = r0.elapsed_time(r1)
        # end to end: obs from pinned host each step, actions back to the host
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record()
        for j in range(args.rollout_steps):
            k = j % nroll
            acts, lp, v = rstep(j, ro_h[k * A:(k + 1) * A])
            acts.cpu()
        q1.record()
        torch.cuda.synchronize()
        qms = q0.elapsed_time(q1)
        # end to end with the compact transfer form (int16 ids): the packed
        # rows cross PCIe and the device expands them into the graph's input
        import ptcg_b200.native as pnative
        pk_h = torch.from_numpy(pnative.obs_pack(s, ro_h.numpy())).pin_memory()
        pk_d = torch.empty(A, pk_h.shape[1], dtype=torch.uint8, device=dev)
        c0_, c1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0_.record()
        for j in range(args.rollout_steps):
            k = j % nroll
            pk_d.copy_(pk_h[k * A:(k + 1) * A], non_blocking=True)
            pol.obs_unpack(pk_d, out=gsrc)
            guni.copy_(uni[j])
            if graph is not None:
                graph.replay()
                acts = gout[0]
            else:
                acts = rstep_static()[0]
            acts.cpu()
        c1_.record()
        torch.cuda.synchronize()
        cms = c0_.elapsed_time(c1_)
        tt = torch.tensor([rms, qms, cms], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        rms, qms, cms = [float(x) for x in tt.cpu()]
        from ptcg_b200.config import forward_flops
        peaks_r, src_r = measured_peaks()
        fl = forward_flops(s, "first")["total"]
        ach = A * args.rollout_steps * fl / (rms / 1e3) / 1e12
        pk = peaks_r.get("bf16_tflops_sustained", 1400.0)
        rollout = {"metric": "rollout forward/sec (config 1)" if args.preset == "c0"
                   else f"rollout forward/sec ({args.preset})", "unit": "obs/s",
                   "value": A * args.rollout_steps * world / (rms / 1e3),
                   "e2e": A * args.rollout_steps * world / (qms / 1e3),
                   "agents_per_gpu": A, "env_steps": args.rollout_steps,
                   "ms_per_env_step": rms / args.rollout_steps,
                   "cuda_graph": graph is not None,
                   "h2d_bytes_per_step": A * s.obs_size * 4, "d2h_bytes_per_step": A * 4,
                   "e2e_compact_obs": {"value": A * args.rollout_steps * world / (cms / 1e3),
                                       "h2d_bytes_per_step": A * int(pk_h.shape[1])},
                   "roofline": {"kernel": "whole rollout forward + sampler (all kernels)",
                                "bound": "tensor", "achieved": ach, "peak": pk,
                                "unit": "TFLOP/s", "frac": ach / pk,
                                "peak_source": f"bf16_tflops_sustained ({src_r})",
                                "gflop_per_obs": fl / 1e9}}
        if graph is None:
            rollout["gpu_launches_per_step"] = (pol.lib.ptcg_launch_count() - l0r) / max(
                1, args.rollout_steps)

    if world > 1:
        pol.set_grad_hook(None)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # --- roofline of the dominant kernel (the GEMM class timed above)
    peaks, src = measured_peaks()
    achieved = kflops / (kms / 1e3) / 1e12 if kms > 0 else 0.0
    peak = peaks.get("bf16_tflops_sustained", 1400.0)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    kname = "gemm_tc (tcgen05)" if timer_mode == 1 else "gemm_simt"
    traffic_note = None
    if os.path.exists(tp):
        # ncu DRAM bytes per launch, captured per preset (a capture of a
        # smaller micro-batch scaled by rows is labelled "scaled")
        t = json.load(open(tp)).get(args.preset, {}).get(kname)
        if t:
            traffic, traffic_note = t["bytes_per_launch"], t["measured"]
    # The class's two roofs: the tensor pipe (FLOPs) and HBM (algorithmic
    # bytes: operands read once, outputs written once).  The bound reported
    # is the roof the class is closer to.
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    hbm_ach = kbytes / (kms / 1e3) / 1e9 if kms > 0 else 0.0
    tens = {"achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak if peak else None,
            "peak_source": f"bf16_tflops_sustained ({src})"}
    hbm = {"achieved": hbm_ach, "peak": hbm_peak, "unit": "GB/s",
           "frac": hbm_ach / hbm_peak if hbm_peak else None,
           "peak_source": f"hbm_gbs copy ({src})",
           "write_only_gbs_measured": write_gbs,
           "algorithmic_bytes_per_launch": kbytes / max(klaunch, 1)}
    main = hbm if (hbm["frac"] or 0) > (tens["frac"] or 0) else tens
    roof = {"kernel": kname, "bound": "hbm" if main is hbm else "tensor",
            "achieved": main["achieved"], "peak": main["peak"], "unit": main["unit"],
            "frac": main["frac"], "traffic": traffic, "traffic_source": traffic_note,
            "peak_source": main["peak_source"],
            "tensor": tens, "hbm": hbm, "launches": klaunch,
            "device_ms": kms, "share_of_step_time": kms / ms if ms else None}

    cpu = None
    if world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        rate, n, med, kind = cpu_step_rate(pkg, s, 64, args.cpu_seconds, threads)
        what = "the reference's torch model" if kind == "reference" else "the CPU oracle port"
        cpu = {"value": rate, "unit": "samples/s", "cores": threads, "kind": kind,
               "sample": f"64-row PPO train step of {what} (forward_train + PPO loss + aux + "
                         f"backward + Adam), median of {n} steps ({med:.2f} s/step)"}
        # the other two CPU figures of the measurement plan: the rollout
        # forward (config 1 shapes) and the scaled config 4 at 16 rows (the
        # port: the reference binds its shapes at import, one per process)
        rr, rn, rmed, rkind = cpu_rollout_rate(pkg, s, 256, args.cpu_seconds / 3, threads)
        cpu["rollout"] = {"value": rr, "unit": "obs/s", "kind": rkind,
                          "sample": f"forward_eval of 256 observations under no_grad, median of "
                                    f"{rn} ({rmed:.2f} s)"}
        s4 = pkg.config.PRESETS["c4"]
        r4, n4, m4, _ = cpu_step_rate(pkg, s4, 16, args.cpu_seconds / 3, threads, port_only=True)
        cpu["c4_train"] = {"value": 1e3 / r4, "unit": "ms/sample", "kind": "port",
                           "sample": f"16-row c4 PPO train step, median of {n4} ({m4:.2f} s/step)"}
    from ptcg_b200.config import train_flops
    flops_exec = train_flops(s, "first")       # what this build runs per sample
    flops_ref = train_flops(s, "all")          # same step with the critic over every row
    line = {
        "metric": metric_name(args.preset),
        "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": arm_config(args, s, world, micro),
        "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "roofline": roof,
        "model_tflops": {"executed": value * flops_exec / world / 1e12,
                         "reference_equivalent": value * flops_ref / world / 1e12,
                         "gflop_per_sample": {"executed": flops_exec / 1e9,
                                              "reference_equivalent": flops_ref / 1e9}},
        "roofline_optimizer": {
            "kernel": "ptcg_adam_step (k_sumsq + k_adam)", "bound": "hbm",
            "achieved": ob / (adam_ms / 1e3) / 1e9, "peak": peaks.get("hbm_gbs"),
            "unit": "GB/s", "frac": ob / (adam_ms / 1e3) / 1e9 / peaks.get("hbm_gbs", 6650.0),
            "traffic": ob, "ms": adam_ms,
            "note": "algorithmic bytes: 32 B per arena float + 2 B per bf16-copied parameter"},
        "rollout": rollout,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
        "weights_identical_across_ranks": ok,
        "grad_buckets": ({"per_step": len(reducer.spans), "cover_arena_once": all(covered)}
                         if reducer is not None else
                         # the library checks at ptcg_dp_init that its spans tile the arena
                         # and, every step, that all of them were reduce-scattered
                         {"exchange": "library (NCCL)", "cover_arena_once": True}
                         if native_dp else None),
        "loss_stats": {"total": float(st[0]), "approx_kl": float(st[5]),
                       "grad_norm": float(st[8])},
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _tc_available(pol):
    return bool(pol.lib.ptcg_tensor_cores())


if __name__ == "__main__":
    main()
