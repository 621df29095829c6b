#!/usr/bin/env python
"""GLAD actor rollout forward benchmark on B200 (qrt full mode: INT8 QuantCNN
+ LET W8A8 linears, dynamic activation scales), env-obs/s at B=4096 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU runs are launched by torchrun, one process per GPU; each rank owns
its own 4096 environments (weak scaling, no data-path collective), the step
time is the max over ranks.

Timing: device time with CUDA events around K graph replays of the fused
forward, inputs rotating over 8 observation buffers (8 x 35.6 MB > 126 MB L2)
resident in HBM. ``e2e`` repeats the step through the public
``InferenceRunner.act_host`` call with the observations copied in from pinned
host memory and the action means copied back every step; two host lanes let the
copy of step k+1 overlap the forward of step k (``serial_value``: one lane).

``--impl reference`` times the reference's own CPU implementation of the
GLAD forward (FP32 eager, rsl_rl actor_critic_encoder.py:342-350, restated in
oracle/cpu_fp32.py) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import copy
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "GLAD actor fwd env-obs/sec & ms/step at B=4096 (INT8 LET), 1/2/4/8 B200"
UNIT = "env-obs/s"
INT8_PATHS = ["actor.0", "actor.2", "actor.4", "actor.6", "actor_proprio_embedding", "query_projector"]
BYTES_PER_ENV_FWD = 8816          # obs read (fp32) + action mean write, fused ideal
MACS_PER_ENV = 2.55e6             # conv1 .. actor MLP (int8 2.02 M + fp16 0.53 M)
OBS_BYTES_PER_ENV = 2175 * 4      # what the front kernel must read per env
# DRAM bytes (read + write) per front_fused_kernel launch per environment, from the ncu
# capture summarised in profiles/front_fused_kernel_glad_b4096.md (35.768 MB read +
# 0.073 MB written at B=4096); traffic grows with the environments processed.
FRONT_DRAM_BYTES_PER_ENV = (35.767552e6 + 0.072704e6) / 4096
N_STAGES = ("absmax", "front", "tail", "actor.0", "actor.2", "actor.4", "actor.6")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20000)
    p.add_argument("--warmup", type=int, default=200)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--batch", type=int, default=4096)
    p.add_argument("--act-mode", choices=("dynamic", "static"), default="dynamic")
    p.add_argument("--nbuf", type=int, default=8)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-conv-chain", action="store_true", help="skip the conv-only (QuantCNN chain) measurement")
    p.add_argument("--no-w4a16", action="store_true", help="skip the W4A16 large-batch measurement")
    p.add_argument("--profile-case", choices=("actor", "chain"), default=None,
                   help="run only this workload for a profiler (warm-up + steps forwards of --batch, "
                        "no graphs, no timing, no JSON line): 'actor' = the fused actor forward, "
                        "'chain' = the QuantCNN chain alone (glad_conv_chain)")
    return p.parse_args()


def rank_info():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


# ---------------------------------------------------------------------------------------------
def _node_of_cpus(cpus) -> list[int]:
    """NUMA nodes holding any of `cpus` (from /sys/devices/system/node)."""
    nodes = []
    base = "/sys/devices/system/node"
    try:
        names = sorted(n for n in os.listdir(base) if n.startswith("node") and n[4:].isdigit())
    except OSError:
        return nodes
    for n in names:
        try:
            spec = open(os.path.join(base, n, "cpulist")).read().strip()
        except OSError:
            continue
        cs = set()
        for part in spec.split(","):
            if "-" in part:
                a, b = part.split("-")
                cs.update(range(int(a), int(b) + 1))
            elif part:
                cs.add(int(part))
        if cs & set(cpus):
            nodes.append(int(n[4:]))
    return nodes


def host_link(device, nbytes: int, barrier, world: int, rank: int, reps: int = 10) -> dict:
    """Where this rank's host buffers and GPU sit, and the host->device copy rate of one
    step's observations (`nbytes` from pinned memory): with the other ranks idle (ranks
    take turns) and with every rank copying at once."""
    import torch.distributed as dist

    info = {"rank": rank}
    try:
        props = torch.cuda.get_device_properties(device)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        info["gpu_pci"] = bus
        info["gpu_numa"] = int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
    except Exception:  # noqa: BLE001
        pass
    try:
        info["cpu_numa"] = _node_of_cpus(sorted(os.sched_getaffinity(0)))
    except Exception:  # noqa: BLE001
        pass
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=device)
    dst.copy_(src, non_blocking=True)

    def rate():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        return nbytes * reps / (a.elapsed_time(b) / 1e3) / 1e9

    alone = None
    for r in range(world):
        barrier()
        if r == rank:
            alone = rate()
    barrier()
    info["h2d_alone_gbs"] = alone
    info["h2d_concurrent_gbs"] = rate()
    barrier()
    if world > 1:
        out = [None] * world
        dist.all_gather_object(out, info)
        return {"ranks": out}
    return {"ranks": [info]}


class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU while the timed work runs."""

    FIELDS = ("clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.lines: list[str] = []
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            gid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.cmd = ["nvidia-smi", "-i", gid, f"--query-gpu={','.join(self.FIELDS)}",
                        "--format=csv,noheader,nounits", "-lms", "50"]
        except Exception:  # noqa: BLE001
            self.cmd = None

    def start(self):
        """Start sampling and wait (up to 3 s) for the first sample, so that the
        sampler's own start-up does not fall inside a short timed region."""
        if not self.cmd:
            return
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return
        self._reader = threading.Thread(target=self._read, daemon=True)
        self._reader.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        time.sleep(0.06)                # one more sample period past the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait(timeout=10)
        self._reader.join(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[3:]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
def build_inference_copy(device, act_mode: str):
    """GLAD seed-0 model -> fp16 copy -> LET calibration (200 Adam steps, 512
    obs from seed 1) -> QuantLinear swap -> QuantCNN -> encoder rewrite, all
    through the package's public API (qrt/integration.py:100-126)."""
    from rl_quant_b200 import calib, calib_cnn_scale, patch_encoder, swap, swap_cnn
    from rl_quant_b200.glad_model import build_glad
    from rl_quant_b200.synthetic import glad_obs

    model = build_glad(seed=0, critic_seed=2, dtype=torch.float32, device=device)
    infer = copy.deepcopy(model).half().eval()
    cal = glad_obs(512, seed=1).half().to(device)
    batches = [{"policy_obs": cal[i * 64:(i + 1) * 64]} for i in range(8)]

    def fn_factory():
        it = iter(batches * 64)
        return lambda: next(it)

    plan = calib.make_plan(infer, INT8_PATHS, obs_fn=fn_factory(), n_calib=8, use_let=True,
                           let_steps=200, act_mode=act_mode, verbose=False, seed=0)
    swap.apply(infer, plan)
    swap_cnn(infer, calib_cnn_scale(infer, fn_factory(), n_batches=8))
    patch_encoder(infer)
    return model, infer.eval()


def bench_conv_chain(device, hbm_peak, conv_w, reps=50):
    """The QuantCNN chain alone (x_nhwc fp16 -> z8 + fp16 local features) at the
    conv-only batch sizes: CUDA-event time per call over rotating buffers larger
    than L2, algorithmic bytes = fp16 input 4,158 B + fp16 features 23,936 B per env."""
    from rl_quant_b200 import _native as N
    from rl_quant_b200.synthetic import glad_obs
    lib = N.load()
    out = {}
    w = None
    for B in (1024, 4096, 16384):
        per_buf = B * (4158 + 23936 + 2992)
        nbuf = max(2, -(-200_000_000 // per_buf))
        x0 = glad_obs(B, seed=77)[:, 96:].half().reshape(B, 21, 33, 3).contiguous().to(device)
        xs = [x0] + [x0.roll(k, 0) for k in range(1, nbuf)]
        feats = [torch.empty(B * 187, 64, dtype=torch.float16, device=device) for _ in range(nbuf)]
        z8s = [torch.empty(B * 187, 16, dtype=torch.int8, device=device) for _ in range(nbuf)]
        if w is None:
            w = conv_w
        for k in range(3):
            N.check(lib.glad_conv_chain(xs[k % nbuf].data_ptr(), B, w, feats[k % nbuf].data_ptr(),
                                        z8s[k % nbuf].data_ptr(), N.stream_handle(device)))
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for k in range(reps):
            lib.glad_conv_chain(xs[k % nbuf].data_ptr(), B, w, feats[k % nbuf].data_ptr(),
                                z8s[k % nbuf].data_ptr(), N.stream_handle(device))
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / reps
        gbs = B * 28094 / (ms / 1e3) / 1e9
        out[str(B)] = {"ms": ms, "env_per_s": B / (ms / 1e3), "achieved_gbs": gbs,
                       "frac_hbm": gbs / hbm_peak, "bytes_per_env": 28094}
        del xs, feats, z8s
    return out


def bench_w4a16(device, hbm_peak, fused, infer, reps=20):
    """The GLAD actor with a W4A16 actor MLP (int4 weights from seed 3, group 64, fp16
    activations) at B = 4096 / 16384 / 65536 per GPU: CUDA-event time per call with the
    obs resident (one buffer per call, each > L2), against 8,816 B/env."""
    import torch.nn as nn
    from rl_quant_b200.synthetic import glad_obs
    from rl_quant_b200.w4a16 import W4A16MLP
    torch.manual_seed(3)
    actor = nn.Sequential(nn.Linear(224, 512), nn.ELU(), nn.Linear(512, 256), nn.ELU(), nn.Linear(256, 128),
                          nn.ELU(), nn.Linear(128, 29)).to(device)
    mlp = W4A16MLP.from_actor(actor)
    out = {}
    for B in (4096, 16384, 65536):
        nbuf = 4 if B == 4096 else 2
        base = glad_obs(B, seed=6006).to(device)
        obs = [base] + [base.roll(k, 0) for k in range(1, nbuf)]
        mean = torch.empty(B, 29, dtype=torch.float32, device=device)
        for k in range(3):
            mlp.actor_forward(fused, obs[k % nbuf], out=mean)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for k in range(reps):
            mlp.actor_forward(fused, obs[k % nbuf], out=mean)
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / reps
        gbs = B * BYTES_PER_ENV_FWD / (ms / 1e3) / 1e9
        out[str(B)] = {"ms": ms, "env_per_s": B / (ms / 1e3), "achieved_gbs": gbs, "frac_hbm": gbs / hbm_peak}
        del obs, base
        torch.cuda.empty_cache()
    return out


def profile_case(args, device, fused):
    """One workload alone, for an ncu capture: --warmup + --steps calls on rotating inputs
    (two buffers), plainly launched so that each kernel is one launch in the list."""
    from rl_quant_b200 import _native as N
    from rl_quant_b200.synthetic import glad_obs
    B, n = args.batch, args.warmup + args.steps
    if args.profile_case == "actor":
        obs = [glad_obs(B, seed=1000 + i).to(device) for i in range(2)]
        mean = torch.empty(B, 29, dtype=torch.float32, device=device)
        for k in range(n):
            fused.run(obs[k % 2], mean)
    else:
        lib = N.load()
        xs = [glad_obs(B, seed=77 + i)[:, 96:].half().reshape(B, 21, 33, 3).contiguous().to(device)
              for i in range(2)]
        feat = torch.empty(B * 187, 64, dtype=torch.float16, device=device)
        z8 = torch.empty(B * 187, 16, dtype=torch.int8, device=device)
        for k in range(n):
            N.check(lib.glad_conv_chain(xs[k % 2].data_ptr(), B, fused.weights().conv, feat.data_ptr(),
                                        z8.data_ptr(), N.stream_handle(device)), "conv chain")
    torch.cuda.synchronize(device)
    print(f"profile case {args.profile_case}: {n} calls at B={B}")


def run_ours(args):
    import torch.distributed as dist

    from rl_quant_b200 import InferenceRunner, _native as N
    from rl_quant_b200.fused import FusedActor, FusedCritic
    from rl_quant_b200.synthetic import glad_obs, glad_obs_pair
    from rl_quant_b200.weight_sync import PackedWeights

    rank, local, world = rank_info()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    B = args.batch
    master, infer = build_inference_copy(device, args.act_mode)
    # every tensor of the inference copy in one device blob: one broadcast per PPO iteration
    packed = PackedWeights(infer)
    fused = FusedActor(infer)
    fused_critic = FusedCritic(infer)
    if fused.act_mode != args.act_mode:
        raise RuntimeError("calibrated model has the wrong act_mode")

    if args.profile_case:
        profile_case(args, device, fused)
        return
    # inputs resident in HBM, rotated so successive steps miss L2
    obs = [glad_obs(B, seed=1000 + 97 * rank + i).to(device) for i in range(args.nbuf)]
    means = [torch.empty(B, 29, dtype=torch.float32, device=device) for _ in range(args.nbuf)]
    for i in range(args.nbuf):          # warm, allocate the workspace outside capture
        fused.run(obs[i], means[i])
    torch.cuda.synchronize()
    graphs = []
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for i in range(args.nbuf):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                fused.run(obs[i], means[i])
            graphs.append(g)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize()
    st = N.c_uint32(0)
    N.check(N.load().glad_workspace_status(fused.workspace(B, device).data_ptr(), st,
                                           N.stream_handle(device)), "device status")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    clocks = ClockSampler(device)
    clocks.start()
    for k in range(args.warmup):
        graphs[k % args.nbuf].replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(args.steps):
        graphs[k % args.nbuf].replay()
    e1.record()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = B * world / (ms_step / 1e3)

    # per-stage device time of the same forward (CUDA events between launches)
    n_st = len(N_STAGES) + 1
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_st)]
    for e in evs:                       # materialise the driver events
        e.record()
    torch.cuda.synchronize(device)
    arr = (N.c_void_p * n_st)(*[e.cuda_event for e in evs])
    stage_ms = [0.0] * len(N_STAGES)
    reps = max(20, min(args.steps, 400))
    N.check(N.load().glad_actor_stage_events(arr, n_st), "stage events")
    try:
        for k in range(reps):
            fused.run(obs[k % args.nbuf], means[k % args.nbuf])
            torch.cuda.synchronize(device)
            for s in range(len(N_STAGES)):
                stage_ms[s] += evs[s].elapsed_time(evs[s + 1])
    finally:
        N.load().glad_actor_stage_events(None, 0)
    stage_ms = [x / reps for x in stage_ms]
    stage_names = list(N_STAGES)
    mlp_fused = N.load().glad_actor_mlp_fused(B, N.ACT_MODES[args.act_mode]) == 1
    if mlp_fused:                       # one kernel for the four MLP layers
        stage_names = stage_names[:3] + ["mlp"]
        stage_ms = stage_ms[:3] + [sum(stage_ms[3:])]
    n_kernels = N.load().glad_actor_kernel_count(B, N.ACT_MODES[args.act_mode])
    if stage_ms[0] < 1e-3:              # the proprio absmax runs inside the front kernel
        stage_names, stage_ms = stage_names[1:], stage_ms[1:]

    # actor + critic forward (one PPO rollout step of both heads)
    n_ac = min(4, args.nbuf)
    pairs = [glad_obs_pair(B, seed=5000 + 97 * rank + i) for i in range(n_ac)]
    a_in = [p[0].to(device) for p in pairs]
    c_in = [p[1].to(device) for p in pairs]
    values = [torch.empty(B, 1, dtype=torch.float32, device=device) for _ in range(n_ac)]
    # the two heads share the scan (as in the reference's benchmark groups): one fused
    # call reads it once; otherwise the actor and critic forwards run back to back
    try:
        from rl_quant_b200.fused import FusedActorCritic, FusedUnsupported
        fused_ac = FusedActorCritic(infer)
    except FusedUnsupported:
        fused_ac = None

    def ac_step(i):
        if fused_ac is not None:
            fused_ac.run(a_in[i], c_in[i], means[i], values[i])
        else:
            fused.run(a_in[i], means[i])
            fused_critic.run(c_in[i], values[i])

    k_ac = max(10, min(args.steps, 1000))

    def time_graphed(step):
        """Capture step(i) for each rotating buffer i, then time k_ac replays (max over ranks)."""
        for i in range(n_ac):
            step(i)
        torch.cuda.synchronize()
        graphs_ = []
        with torch.cuda.stream(side):
            for i in range(n_ac):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    step(i)
                graphs_.append(g)
        torch.cuda.current_stream(device).wait_stream(side)
        for k in range(10):
            graphs_[k % n_ac].replay()
        barrier()
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record()
        for k in range(k_ac):
            graphs_[k % n_ac].replay()
        eb.record()
        barrier()
        ms_ = ea.elapsed_time(eb)
        if world > 1:
            t = torch.tensor([ms_], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_ = float(t.item())
        return ms_

    ms_ac = time_graphed(ac_step)
    ac_value = B * world / (ms_ac / k_ac / 1e3)

    # the whole PPO.act transition (rsl_rl/algorithms/ppo.py:129-140): actor + critic,
    # then the Normal(mean, std) sample and its log-probability (glad_ppo_epilogue)
    ppo = None
    if fused_ac is not None:
        from rl_quant_b200.fused import ppo_epilogue
        std_t = infer.std.detach().float().contiguous()
        rng_t = torch.zeros(2, dtype=torch.int64, device=device)
        acts = [torch.empty(B, 29, dtype=torch.float32, device=device) for _ in range(n_ac)]
        lps = [torch.empty(B, dtype=torch.float32, device=device) for _ in range(n_ac)]
        sgs = [torch.empty(B, 29, dtype=torch.float32, device=device) for _ in range(n_ac)]

        def ppo_step(i):
            fused_ac.run(a_in[i], c_in[i], means[i], values[i])
            ppo_epilogue(means[i], std_t, 1234 + rank, rng_t, acts[i], lps[i], sgs[i])

        ms_ppo = time_graphed(ppo_step)
        ppo = {"value": B * world / (ms_ppo / k_ac / 1e3), "unit": UNIT, "ms_per_step": ms_ppo / k_ac,
               "workload": f"PPO.act transition, B={B} per GPU: fused actor + critic, Normal sample, "
                           "log-prob, sigma (glad_actor_critic_forward + glad_ppo_epilogue)"}

    # end to end through InferenceRunner.act_host with host buffers: every step copies
    # its obs in from pinned host memory and its means back out. Two host lanes: the
    # copy of step k+1 overlaps the forward of step k; one lane: fully serial steps.
    host = [o.cpu().pin_memory() for o in obs[:4]]
    out_host = [torch.empty(B, 29, dtype=torch.float32).pin_memory() for _ in host]
    k_e2e = max(10, min(args.steps, 300))

    def time_e2e(lanes):
        runner = InferenceRunner(infer, mode="manual-graph", host_lanes=lanes)
        for k in range(5):
            runner.act_host(host[k % len(host)], out_host[k % len(host)])
        barrier()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record()
        for k in range(k_e2e):
            runner.act_host(host[k % len(host)], out_host[k % len(host)])
        e3.record()
        barrier()
        ms = e2.elapsed_time(e3)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return B * world / (ms / k_e2e / 1e3)

    e2e_value = time_e2e(2)
    e2e_serial = time_e2e(1)
    links = host_link(device, B * OBS_BYTES_PER_ENV, barrier, world, rank)
    runner = InferenceRunner(infer, mode="manual-graph", with_critic=True)

    # per-iteration weight hand-over: W += 1e-3 N(0,1) on the fp32 master (rank 0,
    # not timed), then [rank 0: graphed cast-copy + requantise] + one NCCL
    # broadcast of the packed blob to every rank (timed, max over ranks)
    n_sync = 30
    gen = torch.Generator(device=device).manual_seed(7)
    sync_ms = 0.0
    for it in range(n_sync + 3):
        if rank == 0:
            with torch.no_grad():
                for p_ in master.parameters():
                    p_.add_(1e-3 * torch.randn(p_.shape, device=device, generator=gen))
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        if rank == 0:
            runner.sync_weights_from(master)
        if world > 1:
            packed.broadcast(src=0)
        s1.record()
        barrier()
        if it >= 3:
            sync_ms += s0.elapsed_time(s1)
    sync_ms /= n_sync
    checks_ok = True
    if world > 1:
        t = torch.tensor([sync_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sync_ms = float(t.item())
        cs = torch.tensor([packed.checksum()], dtype=torch.int64, device=device)
        lo, hi = cs.clone(), cs.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        checks_ok = bool(lo.item() == hi.item())

    if rank == 0:
        peaks = {}
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peaks = json.load(f)
        except OSError:
            pass
        hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
        peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
        tensor_peak = float(peaks.get("bf16_tflops", 1590.0))
        tensor_src = ("measured dense bf16 burst" if "bf16_tflops" in peaks else "fallback dense bf16")
        dom = max(range(len(stage_names)), key=lambda i: stage_ms[i])
        dom_name = stage_names[dom]
        alg_bytes = {"front": OBS_BYTES_PER_ENV * B}.get(dom_name)
        achieved = (alg_bytes / (stage_ms[dom] / 1e3) / 1e9) if alg_bytes else None
        fwd_gbs = BYTES_PER_ENV_FWD * B / (ms_step / 1e3) / 1e9
        tops = MACS_PER_ENV * 2 * B / (ms_step / 1e3) / 1e12
        conv_chain = None
        if world == 1 and not args.no_conv_chain:
            conv_chain = bench_conv_chain(device, hbm_peak, fused.weights().conv)
        w4 = None
        if world == 1 and not args.no_w4a16:
            w4 = bench_w4a16(device, hbm_peak, fused, infer)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            from oracle.cpu_fp32 import time_fp32_forward
            r = time_fp32_forward(batch=256, budget_s=12.0)
            cpu = {"value": r["obs_per_s"], "unit": UNIT, "cores": r["threads"], "kind": "port",
                   "sample": f"FP32 eager GLAD actor forward on the host CPU, B=256 per forward, "
                             f"{r['reps']} forwards back to back after ~1 s of warm-up "
                             f"({r['sec_per_step'] * 1e3:.2f} ms/forward)"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"GLAD actor forward, qrt full mode (INT8 QuantCNN + LET W8A8 "
                                   f"linears, {args.act_mode} s_z), B={B} per GPU",
                       "batch_per_gpu": B, "act_mode": args.act_mode, "obs_dtype": "fp32",
                       "weights": "seed-0 default init, LET calibrated 200 Adam steps on 512 obs (seed 1)",
                       "l2": f"{args.nbuf} rotating obs buffers ({args.nbuf * B * OBS_BYTES_PER_ENV / 1e6:.0f} MB) > 126 MB L2",
                       "launch": f"CUDA graph per step ({n_kernels} kernels: slot clear, front, tail, MLP)"},
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": B * 2175 * 4,
                    "d2h_bytes_per_step": B * 29 * 4, "api": "InferenceRunner.act_host, 2 host lanes",
                    "serial_value": e2e_serial},
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": (achieved / hbm_peak) if achieved else None,
                         "traffic": (FRONT_DRAM_BYTES_PER_ENV * B if dom_name == "front" else None),
                         "peak_source": peak_src,
                         "algorithmic_bytes_per_env": OBS_BYTES_PER_ENV if alg_bytes else None},
            "forward_roofline": {"bytes_per_env": BYTES_PER_ENV_FWD, "achieved_gbs": fwd_gbs,
                                 "frac_hbm": fwd_gbs / hbm_peak, "macs_per_env": MACS_PER_ENV,
                                 "achieved_tops": tops},
            # the forward's 2.55 M MAC per environment (2.02 M int8, 0.53 M fp16) as op/s against the
            # measured dense bf16 GEMM peak (the int8 dense peak is nominally twice that)
            "tensor_roofline": {"achieved": tops, "unit": "TOP/s", "peak": tensor_peak,
                                "frac": tops / tensor_peak if tensor_peak else None,
                                "peak_source": tensor_src},
            "host_links": links["ranks"],
            "stage_ms": dict(zip(stage_names, stage_ms)),
            "actor_critic": {"value": ac_value, "unit": UNIT, "ms_per_step": ms_ac / k_ac,
                             "workload": f"actor + critic forward, B={B} per GPU, {world * B} envs" +
                                         (", one read of the shared scan (glad_actor_critic_forward)"
                                          if fused_ac is not None else "")},
            "ppo_act": ppo,
            "weight_sync": {"ms": sync_ms, "bytes": packed.nbytes,
                            "collective": "nccl broadcast of one packed blob" if world > 1 else "none (1 GPU)",
                            "steps": "cast-copy fp32 master -> fp16 copy + requantise (one CUDA graph) + broadcast",
                            "ranks_identical": checks_ok},
            "conv_chain": ({"workload": "QuantCNN chain alone (glad_conv_chain): x_nhwc fp16 -> z8 + fp16 "
                                        "local features; rotating buffers > L2; events per call",
                            "per_batch": conv_chain} if conv_chain else None),
            "w4a16": ({"workload": "GLAD actor, INT8 encoder + W4A16 actor MLP (int4 weights from seed 3, "
                                   "group 64, fp16 activations), dynamic s_z, obs resident, events per call",
                       "per_batch": w4} if w4 else None),
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * n_kernels,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        del graphs                      # (the timing helpers' graphs are released on return)
        dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the reference's FP32 eager forward on the host cores, rank 0
    only. Each step is a bounded sample of the workload: as many back-to-back B=256
    forwards as take about 0.25 s; W warm-up steps (at least 3), then K timed steps;
    the value is the env-obs/s of the whole timed region."""
    rank, _, world = rank_info()
    if rank != 0:
        return
    from oracle.cpu_fp32 import Fp32Forward

    f = Fp32Forward(batch=256)
    per_step = f.forwards_for(0.25)
    warm = max(3, args.warmup)
    steps = args.steps
    if (warm + steps) * 0.25 > 150.0:          # keep the arm within a few minutes
        warm, steps = min(warm, 20), max(3, min(steps, 580))
    for _ in range(warm):
        f.run(per_step)
    dt = sum(f.run(per_step) for _ in range(steps))
    v = f.batch * per_step * steps / dt
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"GLAD actor forward (FP32 eager, reference CPU path): each step "
                               f"{per_step} forwards of B=256 from the B={args.batch} workload",
                   "batch_per_forward": 256, "forwards_per_step": per_step},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": f.threads, "kind": "port",
                         "sample": f"{steps} steps x {per_step} forwards of B=256 after {warm} warm-up steps"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)
