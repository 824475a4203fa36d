#!/usr/bin/env python3
"""Benchmark of the B200 Flow decoder hot path.

Workload (the configuration the metric is quoted on at
1/2/4/8 GPUs): per GPU, 64 independent utterances with lengths uniform in
[100, 1500] mel frames (seed 3), each with its own N(0,1) mu/spks/noise and a
prompt cond over its first 20% of frames, decoded by the 10-step cosine CFM
Euler solver with CFG pairing (batch 2 per utterance) through the 22-block
DiT, key-padding semantics (utterances packed without padding).  Weights are
seeded random N(0, 0.02) of the real architecture (no checkpoint offline).

One step = one full 10-step CFG decode of the 64-utterance set.  At N GPUs
the set is split across the ranks by decode cost (larynx_b200.shard: LPT over
a device-time model, then a local search), each rank decodes its shard, and
`value` = the set's mel frames / max-over-ranks device time (strong scaling:
the work is fixed as N grows), with inputs resident in HBM
(lx_flow_decode_device); `e2e` = the same through the host-buffer C-ABI call
lx_flow_decode (pinned inputs, H2D + compute + D2H of the mel every step).
There is no collective on the data path (barriers and the timing max only).
`cfg3_weak` (N > 1) is the weak-scaling view: every rank decodes the whole
set.

`--impl reference` times the reference's CPU path on the host cores.  The
reference's own CPU engine (GGML, LARYNX_BACKEND=cpu) cannot be built (ggml is
an un-vendored submodule), so a float32 restatement of the reference's Flow
model in torch CPU operators (oracle/flow_cpu.py: checked against the numpy
oracle, which is pinned to the reference's golden vectors; it runs at the
speed of the reference's own PyTorch model on the same cores) runs in its
place on every host core, one Euler step of one config-3 utterance per step
(a 10-step decode is ten such forwards, so frames / (10 x step time) is its
throughput), the utterances taken from the set in a fixed order that mixes
short and long ones.
"""

import argparse
import datetime
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "Flow mel-frames/s (10-step CFG)"
UNIT = "mel-frames/s"
N_UTT = 64
REF_SAMPLE_STRIDE = 23   # coprime to 64: any run of steps visits lengths from the whole range


def cfg3_lengths(n=N_UTT):
    return np.random.default_rng(3).integers(100, 1501, n).astype(np.int32)


def cfg3_inputs(lengths, seed):
    rng = np.random.default_rng(seed)
    tot = int(np.sum(lengths))
    mu = rng.standard_normal(tot * 80, dtype=np.float32)
    noise = rng.standard_normal(tot * 80, dtype=np.float32)
    spks = rng.standard_normal((len(lengths), 80), dtype=np.float32)
    cond = np.zeros(tot * 80, np.float32)
    off = 0
    for L in lengths:
        L = int(L)
        blk = cond[off:off + 80 * L].reshape(80, L)
        p = int(0.2 * L)
        blk[:, :p] = rng.standard_normal((80, p), dtype=np.float32)
        off += 80 * L
    return mu, cond, spks, noise


def subset(lengths, arrays, idx):
    """The utterances `idx` of a set laid out as concat_u [80][T_u] (mu, cond,
    noise) and [U][80] (spks)."""
    off = np.concatenate([[0], np.cumsum(np.asarray(lengths, np.int64) * 80)])
    mu, cond, spks, noise = arrays
    cat = lambda a: np.ascontiguousarray(np.concatenate([a[off[i]:off[i + 1]] for i in idx]))
    return np.asarray(lengths)[idx], (cat(mu), cat(cond), np.ascontiguousarray(spks[idx]), cat(noise))


def config_block(n_gpus, lengths):
    return {"workload": f"cfg3: one set of {len(lengths)} utterances, T~U[100,1500] frames (seed 3), "
                        "10-step cosine CFM Euler, CFG batch 2, key-padding (packed varlen), dim 1024 x 22 blocks",
            "model": "CosyVoice3 Flow DiT (22 blocks, dim 1024, 16 heads x 64, FF 2048)",
            "global_batch": int(len(lengths)), "seq_len": "100-1500 frames",
            "frames": int(np.sum(lengths)),
            "parallelism": f"dp{n_gpus} (the set sharded across GPUs by decode cost, no collectives)",
            "l2": "inputs larger than L2 (bf16 weights 378 MB + >1 GB activations per step)"}


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.f.seek(0)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        busy = [v for v in sm if v > 0.5 * mx] or sm
        return {"sm_mhz": float(np.median(busy)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# roofline bookkeeping
# ---------------------------------------------------------------------------
def algorithmic_per_launch(cls, lengths):
    """(quantity, unit, bound) per launch of a kernel class for the batch."""
    tok = 2 * int(np.sum(lengths))           # CFG rows
    sq = 2 * float(np.sum(np.asarray(lengths, np.float64) ** 2))
    D, F, M = 1024, 2048, 80
    flops = {"qkv_gemm": 2.0 * tok * 3 * D * D, "out_gemm": 2.0 * tok * D * D, "ff1_gemm": 2.0 * tok * F * D,
             "ff2_gemm": 2.0 * tok * D * F, "attention": 4.0 * D * sq, "in_proj": 2.0 * tok * D * M,
             "conv_pos": 2.0 * tok * D * 64 * 31, "proj_out_gemm": 2.0 * tok * M * D}
    if cls in flops:
        return flops[cls], "TFLOP/s", "tensor"
    if cls == "adaln":
        return tok * D * (4 + 2) + 2 * D * 4, "GB/s", "hbm"
    if cls == "euler":
        return int(np.sum(lengths)) * M * (4 * 4 + 2 * 2), "GB/s", "hbm"
    return None, None, None


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm": float(d["hbm_gbs"]), "tensor": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "tensor_burst": float(d["bf16_tflops"]),
                "sustained_mhz": (d.get("clocks_under_load") or {}).get("sm_mhz_median"),
                "src": "measured (MEASURED_PEAKS.json; sustained bf16 for kernels inside the long step)"}
    return {"hbm": 6650.0, "tensor": 1400.0, "tensor_burst": 1590.0, "sustained_mhz": 1300.0,
            "src": "fallback (6.65 TB/s, 1.59 PF/s burst, 1.4 PF/s sustained)"}


def load_traffic():
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return {}
    return {}


# ---------------------------------------------------------------------------
# CPU arms (the reference's algorithm restated in numpy: oracle/)
# ---------------------------------------------------------------------------
_CPU_MODEL = {}


def cpu_model(W):
    """The multithreaded CPU restatement (oracle/flow_cpu.py) over weights W."""
    if id(W) not in _CPU_MODEL:
        from oracle.flow_cpu import FlowCPU
        _CPU_MODEL.clear()
        _CPU_MODEL[id(W)] = FlowCPU(W)
    return _CPU_MODEL[id(W)]


def cpu_euler_step(W, T, seed):
    """One CFG Euler step (the DiT on the [cond; uncond] rows) of a T-frame
    utterance on the host; returns its wall time."""
    import torch
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, 80, T), dtype=np.float32)
    mu = rng.standard_normal((1, 80, T), dtype=np.float32)
    spk = rng.standard_normal((1, 80), dtype=np.float32)
    cond = np.zeros((1, 80, T), np.float32)
    cond[:, :, :int(0.2 * T)] = rng.standard_normal((1, 80, int(0.2 * T)), dtype=np.float32)
    z = np.zeros_like(mu)
    args = [torch.from_numpy(np.ascontiguousarray(a)) for a in
            (np.concatenate([x, x]), np.concatenate([mu, z]), np.full(2, 0.3, np.float32),
             np.concatenate([spk, np.zeros_like(spk)]), np.concatenate([cond, np.zeros_like(cond)]))]
    m = cpu_model(W)
    t0 = time.perf_counter()
    with torch.inference_mode():
        m.dit_forward(*args)
    return time.perf_counter() - t0


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_sample(W, n, first):
    """`n` samples from the config-3 set: one Euler step of utterance
    order[(first + i) % 64] each.  Returns (frames / s of the 10-step decode,
    the lengths visited)."""
    lengths = np.sort(cfg3_lengths())
    visit = [int(lengths[((first + i) * REF_SAMPLE_STRIDE) % len(lengths)]) for i in range(n)]
    secs = [cpu_euler_step(W, T, 1000 + first + i) for i, T in enumerate(visit)]
    return float(np.sum(visit)) / (10.0 * float(np.sum(secs))), visit


def cpu_threads():
    """Give the CPU arm every host core (torchrun sets OMP_NUM_THREADS=1)."""
    import torch
    n = cpu_cores()
    torch.set_num_threads(n)
    return n


CPU_SAMPLE_ABOUT = ("one CFG Euler step (DiT forward on the cond + uncond rows) of one config-3 utterance per "
                    "sample, utterances from the 64-utterance set in a fixed order mixing short and long ones; "
                    "frames / (10 x time), a 10-step decode being ten such forwards; fp32 restatement of the "
                    "reference's Flow model in torch CPU operators on every host core (oracle/flow_cpu.py, "
                    "checked against the numpy oracle; the same speed as the reference's own PyTorch model on "
                    "the same cores); the reference's GGML CPU engine is unavailable (ggml not vendored)")


def run_reference(args):
    """The reference arm: rank 0 only; other ranks exit without work."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from oracle import flow_oracle as fo
    cores = cpu_threads()
    W = fo.synth_weights(seed=0, std=0.02)
    cpu_sample(W, args.warmup, 64)
    t0 = time.perf_counter()
    value, visit = cpu_sample(W, args.steps, 0)
    wall = time.perf_counter() - t0
    sample = f"{CPU_SAMPLE_ABOUT}; {args.steps} samples, {int(np.sum(visit))} frames"
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_block(args.gpus, cfg3_lengths()),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# BASELINE config 1 (fused-op microbench) and config 4 (streaming chunks)
# ---------------------------------------------------------------------------
CFG1_OPS = (("adaln", 0), ("gate_residual", 1), ("rotary", 2), ("gelu_tanh", 3))


def bench_cfg1(dev, stream, rows=2000, sets=16, reps=20):
    """Standalone fused ops on [2000, 1024] (seed 1, mods N(0, 0.5)), fp32 in
    and bf16 in, fp32 out; `sets` rotating buffer sets (> L2) so every launch
    reads HBM.  GB/s = algorithmic bytes / device time per launch."""
    import torch
    from larynx_b200 import flow
    g = torch.Generator(device="cpu").manual_seed(1)
    D = 1024
    mods = (torch.randn(2, 6 * D, generator=g) * 0.5).to(dev)
    shift, scale, gate = mods[0, :D].contiguous(), mods[0, D:2 * D].contiguous(), mods[1, :D].contiguous()
    pos = (torch.arange(rows, dtype=torch.int32) % 1500).to(dev)
    peak = load_peaks()["hbm"]
    out = {}
    res = [torch.randn(rows, D, generator=g).to(dev) for _ in range(sets)]  # fp32 residual (gate_residual)
    ys = [torch.empty(rows, D, device=dev) for _ in range(sets)]            # fp32 outputs
    for bf in (False, True):
        xs = [torch.randn(rows, D, generator=g).to(dev) for _ in range(sets)]
        if bf:
            xs = [x.to(torch.bfloat16) for x in xs]
        sin = 2 if bf else 4
        for name, op in CFG1_OPS:
            if op == 1:  # x_res += gate * branch: residual read + write, branch read
                nbytes = rows * D * (8 + sin)
                launch = lambda i: flow.op(1, bf, rows, res[i % sets].data_ptr(), xs[i % sets].data_ptr(),
                                           gate_ptr=gate.data_ptr(), stream=stream.cuda_stream)
            else:
                nbytes = rows * D * (sin + 4)
                launch = lambda i, op=op: flow.op(op, bf, rows, xs[i % sets].data_ptr(), ys[i % sets].data_ptr(),
                                                  shift_ptr=shift.data_ptr(), scale_ptr=scale.data_ptr(),
                                                  pos_ptr=pos.data_ptr(), stream=stream.cuda_stream)
            # the launches are captured in a CUDA graph, as the decode runs
            # them, so the per-launch host overhead is not in the figure
            with torch.cuda.stream(stream):
                for i in range(sets):
                    launch(i)
                stream.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(sets * reps):
                        launch(i)
                graph.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                graph.replay()
                e1.record(stream)
                stream.synchronize()
                del graph
            us = e0.elapsed_time(e1) * 1e3 / (sets * reps)
            gbs = nbytes / (us * 1e-6) / 1e9
            out[f"{name}_{'bf16' if bf else 'f32'}_in"] = {"us": round(us, 2), "GB/s": round(gbs, 1),
                                                             "frac_of_hbm": round(gbs / peak, 3)}
    out["_about"] = (f"[{rows},1024] per launch, {sets} rotating buffer sets (> L2), fp32 out, {sets * reps} "
                     "launches in one CUDA graph; gate_residual updates an fp32 residual with an fp32/bf16 "
                     "branch; frac of the measured HBM copy bandwidth")
    return out


def bench_cfg4(dec, dev, stream, streams=256, iters=3):
    """256 streams, each one 50-frame chunk + 6-frame lookahead after
    ctx ~ 50 * U{0..10} frames of context (seed 4), block-causal chunk mask
    (chunk 50), 10-step CFG decode of every stream's whole sequence (stateless
    recompute).  Counts the 50 emitted frames per stream."""
    import torch
    out = {}
    rng = np.random.default_rng(4)
    cases = {"mixed_ctx": (50 * rng.integers(0, 11, streams) + 56).astype(np.int32),
             "worst_ctx500": np.full(streams, 556, np.int32)}
    for name, L in cases.items():
        mu, cond, spks, noise = cfg3_inputs(L, seed=4)
        t = [torch.from_numpy(a).to(dev) for a in (mu, cond, spks, noise)]
        o = torch.empty_like(t[0])
        times = []
        with torch.cuda.stream(stream):
            for i in range(iters + 2):
                a0 = torch.cuda.Event(enable_timing=True)
                a1 = torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                dec.decode_device(L, t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(),
                                  o.data_ptr(), chunk=50, stream=stream.cuda_stream)
                a1.record(stream)
                stream.synchronize()
                if i >= 2:
                    times.append(a0.elapsed_time(a1))
        ms = float(np.median(times))
        out[name] = {"ms_per_chunk_step": round(ms, 3), "emitted_frames_per_s": round(streams * 50 / (ms * 1e-3), 1),
                     "frames_decoded_per_s": round(float(L.sum()) / (ms * 1e-3), 1),
                     "frames_per_batch": int(L.sum())}
    return out


def bench_hift(dev, T=1000, iters=5, with_cpu=True):
    """HiFT vocoder (the stage after the Flow decoder) on one 20 s utterance:
    mel [80][T] in HBM -> 24 kHz audio, device-timed, synthetic weights and
    source bank.  The conv network runs in float32 on the CUDA cores; its
    FLOP rate is reported against the nominal FP32 CUDA-core peak."""
    import tempfile
    import torch
    from larynx_b200.hift import HiftVocoder, conv_flops
    from larynx_b200.hift_weights import synthetic_source, write_source_asset, write_synthetic_hift_gguf
    d = tempfile.mkdtemp(prefix="hift_bench_")
    gp, sp = os.path.join(d, "hift.gguf"), os.path.join(d, "hift_source.bin")
    write_synthetic_hift_gguf(gp, seed=0)
    ri, bank = synthetic_source(0)
    write_source_asset(sp, ri, bank)
    del bank
    v = HiftVocoder(dev.index or 0)
    ok = v.load(gp) and v.load_source(sp)
    for p in (gp, sp):
        os.remove(p)
    os.rmdir(d)
    if not ok:
        return {"error": v.last_error}
    s = torch.cuda.Stream(dev)
    mel = torch.randn(80, T, device=dev, generator=torch.Generator(dev).manual_seed(5))
    audio = torch.empty(T * 480, device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    for _ in range(3):
        v.vocode_device(mel.data_ptr(), T, audio.data_ptr(), s.cuda_stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        v.vocode_device(mel.data_ptr(), T, audio.data_ptr(), s.cuda_stream)
    e1.record(s)
    s.synchronize()
    ms = e0.elapsed_time(e1) / iters
    v.close()
    fl = conv_flops(T)
    bf16 = load_peaks()["tensor"]
    ach = fl / (ms * 1e-3) / 1e12
    cpu = None
    if with_cpu:
        # the oracle port on the host cores (the reference's own HiFT runs its
        # conv network through GGML, which is not buildable here)
        from larynx_b200.hift_weights import synthetic_weights
        from oracle import hift_oracle as ho
        Tc = 100
        w = synthetic_weights(0)
        ri, bank = synthetic_source(1, Tc * 480)
        melc = np.random.default_rng(6).standard_normal((80, Tc)).astype(np.float32)
        t0 = time.perf_counter()
        ho.vocode(melc, ri, bank, w)
        sec = time.perf_counter() - t0
        cpu = {"value": round(Tc / sec, 1), "unit": "mel-frames/s", "cores": cpu_cores(), "kind": "port",
               "sample": f"1 utterance x {Tc} frames (numpy restatement of the reference's HiFT, oracle/)"}
    return {"T_frames": T, "audio_s": T * 480 / 24000, "ms": round(ms, 3),
            "mel_frames_per_s": round(T / (ms * 1e-3), 1), "rtf": (ms * 1e-3) / (T * 480 / 24000),
            "conv_tflops_fp32_equiv": round(ach, 2),
            "ceiling_tflops": round(bf16 / 3, 1), "frac_of_ceiling": round(ach / (bf16 / 3), 3),
            "cpu_baseline": cpu,
            "finite": bool(torch.isfinite(audio).all().item()),
            "about": "whole vocoder (f0 fp64, SineGen2, STFT, conv network, ISTFT) per call; the convs with "
                     "64-multiple channel counts run on tcgen05 with a 3-term bf16 split (3 bf16 products per "
                     "fp32-equivalent product), so their ceiling is the measured sustained bf16 peak / 3; "
                     "conv_tflops_fp32_equiv = conv-network FLOPs / whole-call time"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist_on = world > 1
    # stdout carries exactly one JSON line: anything a library prints there
    # (e.g. NCCL's version banner) is sent to stderr instead
    sys.stdout.flush()
    json_fd = os.dup(1)
    os.dup2(2, 1)
    if dist_on:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist_on:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if not dist_on:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from larynx_b200 import FlowDecoder
    from larynx_b200.weights import write_synthetic_gguf

    wdir = os.environ.get("LX_BENCH_DIR", tempfile.gettempdir())
    gguf = os.path.join(wdir, "lx_bench_flow_synth.gguf")
    if rank == 0 and not os.path.exists(gguf):
        write_synthetic_gguf(gguf + ".tmp", seed=0, std=0.02)
        os.replace(gguf + ".tmp", gguf)
    barrier()
    dec = FlowDecoder(local)
    if not dec.load(gguf):
        raise SystemExit(f"load failed: {dec.last_error}")

    # the config-3 set; this rank decodes its shard (the whole set at N = 1)
    all_lengths = cfg3_lengths(args.utts)
    all_arrays = cfg3_inputs(all_lengths, seed=3000)
    total_frames = int(all_lengths.sum())
    if dist_on:
        from larynx_b200 import shard
        mine = shard.lpt_partition(all_lengths, world)[rank]
    else:
        mine = np.arange(len(all_lengths))
    lengths, (mu, cond, spks, noise) = subset(all_lengths, all_arrays, mine)
    tot = int(lengths.sum())
    dev = torch.device("cuda", local)
    d_mu = torch.from_numpy(mu).to(dev)
    d_cond = torch.from_numpy(cond).to(dev)
    d_spk = torch.from_numpy(spks).to(dev)
    d_noise = torch.from_numpy(noise).to(dev)
    d_out = torch.empty_like(d_mu)
    stream = torch.cuda.Stream(device=dev)

    def step():
        dec.decode_device(lengths, d_mu.data_ptr(), d_cond.data_ptr(), d_spk.data_ptr(), d_noise.data_ptr(),
                          d_out.data_ptr(), stream=stream.cuda_stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        clocks = Clocks()
        if rank == 0:
            clocks.start()
        barrier()
        n0 = dec.launch_count
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        stream.synchronize()
        barrier()
        launches = dec.launch_count - n0
        clk = clocks.stop() if rank == 0 else None
        local_ms = e0.elapsed_time(e1)
        ms = max_over_ranks(local_ms)
    finite = bool(torch.isfinite(d_out).all().item())

    # e2e through the host-buffer C-ABI call, pinned inputs and output
    e2e = None
    if not args.no_e2e:
        pin = lambda a: torch.from_numpy(a).pin_memory()
        p_mu, p_cond, p_spk, p_noise = pin(mu), pin(cond), pin(spks), pin(noise)
        p_out = torch.empty(tot * 80, dtype=torch.float32).pin_memory()
        args_np = (p_mu.numpy(), p_cond.numpy(), p_spk.numpy(), p_noise.numpy(), p_out.numpy())

        def e2e_step():
            dec.decode(lengths, args_np[0], args_np[1], args_np[2], noise=args_np[3], out=args_np[4])

        for _ in range(max(1, min(args.warmup, 2))):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        barrier()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": total_frames * args.steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": int(mu.nbytes + cond.nbytes + spks.nbytes + noise.nbytes),
               "d2h_bytes_per_step": int(tot * 80 * 4), "ms_per_step": e2e_s / args.steps * 1e3,
               "bytes_note": "per rank (this rank's shard)" if dist_on else "whole set",
               "api": "lx_flow_decode (host buffers)"}

    # per-kernel-class device times (CUDA events around every launch, no graph)
    with torch.cuda.stream(stream):
        prof = dec.profile_decode(lengths, d_mu.data_ptr(), d_cond.data_ptr(), d_spk.data_ptr(), d_noise.data_ptr(),
                                  d_out.data_ptr(), stream=stream.cuda_stream)
    peaks = load_peaks()
    traffic = load_traffic()
    # The dominant kernel is the tcgen05 projection GEMM (k_gemm2: one kernel
    # template, launched for QKV, out, FF1 and FF2 of every block): its time
    # share exceeds any other kernel's.  achieved = algorithmic FLOPs of its
    # launches / their summed device time (= per-launch average).
    gem = ("qkv_gemm", "out_gemm", "ff1_gemm", "ff2_gemm")
    g_ms = sum(prof[k][0] for k in gem)
    g_n = sum(prof[k][1] for k in gem)
    g_fl = sum(algorithmic_per_launch(k, lengths)[0] * prof[k][1] for k in gem)
    achieved = g_fl / (g_ms * 1e-3) / 1e12
    # ncu traffic of a smaller capture, scaled to this rank's packed rows
    # (two CFG sequences per utterance, each padded to 8 rows)
    rows = int(2 * np.sum((np.asarray(lengths) + 7) // 8 * 8))
    rs = rows / float(traffic.get("rows_bench", rows) or rows)
    tr = [traffic.get(k, {}).get("bytes_per_launch_scaled") for k in gem]
    traffic_pl = (sum(t * rs * prof[k][1] for t, k in zip(tr, gem)) / g_n) if all(tr) else None
    alg_bytes = None
    if traffic.get("algorithmic_bytes_per_launch"):
        ab = traffic["algorithmic_bytes_per_launch"]
        alg_bytes = sum(ab[k] * rs * prof[k][1] for k in gem) / g_n if all(k in ab for k in gem) else None
    roofline = {"kernel": "k_gemm2 (tcgen05 CTA-pair GEMM: QKV, out, FF1, FF2 projections)", "bound": "tensor",
                "achieved": achieved, "peak": peaks["tensor"], "unit": "TFLOP/s", "frac": achieved / peaks["tensor"],
                "traffic": traffic_pl, "traffic_unit": "bytes per launch (ncu dram read+write, scaled)",
                "algorithmic_bytes_per_launch": alg_bytes, "launch_ms": g_ms / max(1, g_n),
                "launches_per_step": g_n, "share_of_step": g_ms / sum(v[0] for v in prof.values()),
                "peak_source": peaks["src"], "note": "frac of measured sustained bf16 peak",
                "frac_of_burst": achieved / peaks["tensor_burst"], "peak_burst": peaks["tensor_burst"],
                "sm_mhz_during_bench": (clk or {}).get("sm_mhz"), "sm_mhz_during_peak_measurement":
                    peaks["sustained_mhz"],
                "clock_note": "the sustained peak was measured at a lower SM clock than this step ran at; "
                              "frac_of_burst is the clock-neutral bound"}
    # attention: its bound at head dim 64 is the exponential / softmax issue
    # rate, not the tensor pipe; report both views
    a_ms, a_n = prof["attention"]
    a_fl = algorithmic_per_launch("attention", lengths)[0]
    sq_pad = 2.0 * float(np.sum(((np.asarray(lengths) + 127) // 128 * 128).astype(np.float64) ** 2)) * 16
    mhz = (clk or {}).get("sm_mhz") or 1965.0
    mufu_peak = 16 * 148 * mhz * 1e6  # ex2 per second: 16 per clock per SM
    attn = {"achieved_tflops": a_fl / (a_ms / a_n * 1e-3) / 1e12,
            "frac_of_tensor_peak": a_fl / (a_ms / a_n * 1e-3) / 1e12 / peaks["tensor"],
            "exp_per_s": sq_pad / (a_ms / a_n * 1e-3), "mufu_peak_per_s_at_sampled_clock": mufu_peak,
            "frac_of_mufu": sq_pad / (a_ms / a_n * 1e-3) / mufu_peak, "launch_ms": a_ms / a_n,
            "share_of_step": a_ms / sum(v[0] for v in prof.values())}
    breakdown = {}
    for k, (t, n) in prof.items():
        if n == 0:
            continue
        qq, u, b = algorithmic_per_launch(k, lengths)
        e = {"ms_total": round(t, 3), "launches": n, "share": round(t / sum(v[0] for v in prof.values()), 4)}
        if qq:
            a = (qq / (t / n * 1e-3)) / (1e12 if u == "TFLOP/s" else 1e9)
            e.update({"achieved": round(a, 1), "unit": u, "frac_of_peak": round(a / peaks[b], 3)})
        breakdown[k] = e

    # single long utterance latency on this GPU
    extra = {}
    if not args.no_cfg2:
        L2 = np.array([1000], np.int32)
        m2, c2, s2, n2 = cfg3_inputs(L2, seed=2)
        t2 = [torch.from_numpy(a).to(dev) for a in (m2, c2, s2, n2)]
        o2 = torch.empty_like(t2[0])
        times = []
        with torch.cuda.stream(stream):
            for i in range(8):
                a0 = torch.cuda.Event(enable_timing=True)
                a1 = torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                dec.decode_device(L2, t2[0].data_ptr(), t2[1].data_ptr(), t2[2].data_ptr(), t2[3].data_ptr(),
                                  o2.data_ptr(), stream=stream.cuda_stream)
                a1.record(stream)
                stream.synchronize()
                if i >= 3:
                    times.append(a0.elapsed_time(a1))
        extra["cfg2_T1000_latency_ms"] = float(np.median(times))
        extra["cfg2_frames_per_s"] = 1000.0 / (float(np.median(times)) * 1e-3)

    if dist_on:
        # weak-scaling view: every rank decodes the whole 64-utterance set
        wl, wa = all_lengths, all_arrays
        tw = [torch.from_numpy(a).to(dev) for a in wa]
        ow = torch.empty_like(tw[0])
        with torch.cuda.stream(stream):
            for i in range(3):
                if i == 2:
                    barrier()
                    b0 = torch.cuda.Event(enable_timing=True)
                    b1 = torch.cuda.Event(enable_timing=True)
                    b0.record(stream)
                dec.decode_device(wl, tw[0].data_ptr(), tw[1].data_ptr(), tw[2].data_ptr(), tw[3].data_ptr(),
                                  ow.data_ptr(), stream=stream.cuda_stream)
            b1.record(stream)
            stream.synchronize()
        wms = max_over_ranks(b0.elapsed_time(b1))
        extra["cfg3_weak"] = {"value": world * float(total_frames) / (wms * 1e-3), "unit": UNIT, "ms": wms,
                              "about": "every rank decodes the whole 64-utterance set (weak scaling)"}
        del tw, ow
        per_rank = torch.zeros(world, 2, dtype=torch.float64, device=dev)
        per_rank[rank, 0] = local_ms / args.steps
        per_rank[rank, 1] = tot
        dist.all_reduce(per_rank)
        pr = per_rank.cpu().numpy()
        extra["shards"] = {"ms_per_step_by_rank": [round(float(v), 2) for v in pr[:, 0]],
                           "frames_by_rank": [int(v) for v in pr[:, 1]],
                           "balance_max_over_mean": float(pr[:, 0].max() / pr[:, 0].mean()),
                           "partition": "larynx_b200.shard.lpt_partition (LPT + local search on a device-time model)"}
    if not args.no_cfg1:
        extra["cfg1_ops"] = bench_cfg1(dev, stream)
    if not args.no_cfg4:
        extra["cfg4_stream"] = bench_cfg4(dec, dev, stream)
    if world == 1 and not args.no_hift:
        extra["hift"] = bench_hift(dev, with_cpu=not args.no_cpu)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import flow_oracle as fo
        cores = cpu_threads()
        W = fo.synth_weights(seed=0, std=0.02)
        cpu_euler_step(W, 48, 7)  # warm the BLAS threads
        v, visit = cpu_sample(W, 3, 0)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{CPU_SAMPLE_ABOUT}; {len(visit)} samples, {int(np.sum(visit))} frames"}

    if rank == 0:
        value = total_frames * args.steps / (ms * 1e-3)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random weights and inputs)",
                "config": config_block(world, all_lengths),
                "rtf": (ms / args.steps * 1e-3) / (total_frames / 50.0),
                "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline, "cpu_baseline": cpu,
                "clocks": clk, "kernels": breakdown, "attention": attn, "finite": finite, **extra}
        sys.stdout.flush()
        os.write(json_fd, (json.dumps(line) + "\n").encode())
    dec.close()
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--utts", type=int, default=N_UTT)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-cfg2", action="store_true")
    ap.add_argument("--no-cfg1", action="store_true")
    ap.add_argument("--no-cfg4", action="store_true")
    ap.add_argument("--no-hift", action="store_true")
    ap.add_argument("--only-hift", action="store_true",
                    help="time only the HiFT vocoder (one 20 s utterance) and print its JSON object")
    ap.add_argument("--only-cfg1", action="store_true",
                    help="time only the config-1 fused-op microbench and print its JSON object")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.only_hift:
        import torch
        print(json.dumps(bench_hift(torch.device("cuda", 0), with_cpu=not args.no_cpu)))
        return
    if args.only_cfg1:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(bench_cfg1(dev, torch.cuda.Stream(device=dev))))
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
