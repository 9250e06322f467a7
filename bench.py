"""Batch RTFx of the FastConformer encoder hot path on B200.

One step = one batch of synthetic utterances through the hot path (log-mel
front end, dw-striding subsampling, all conformer layers) of the workload's
model. The default workload is the north star's: the 0.6B-class encoder with
f16 weights on a GLOBAL batch of 64 clips of U(2, 35) s (BASELINE
configuration 3's batch). `value` is audio-seconds per second with the PCM
already in HBM (the device-resident C-ABI entry); `e2e` is the same metric
through the public host-buffer C-ABI call (pinned PCM in, encoder output back
to host memory, copies inside the timed region).

Multi-GPU: one process per GPU (torchrun). The global batch is sharded by
whole utterances with the library's own LPT planner (pkc_shard_plan): every
rank encodes its share of the same 64 clips, so the total work is fixed as N
grows -> "scaling": "strong". No collective on the data path; timing is CUDA
events on the launching stream, max over ranks (NCCL all-reduce of the
figures after the timed region).

`--impl reference` times the reference's CPU path on the host cores instead:
parakeet.cpp's ggml encoder cannot be built here (its ggml dependency is absent
from the checkout), so the encoder runs as the CPU restatement in oracle/
(numpy in float32, every BLAS thread) and the mel front end as parakeet.cpp's
own MelFrontend compiled from its sources (oracle/_ref) when present.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "parakeet.cpp_b200", "python"), os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "batch RTFx (audio-s/s) at 1/2/4/8 B200; per-kernel % of HBM/tensor peak"
UNIT = "audio-s/s"
DEFAULT_CONFIG = "c2_0.6b_f16"
# global batch of each workload (split across the ranks): the north star's
# batch 64 for the 0.6B f16 / q8_0 models, the configuration's own otherwise
GLOBAL_BATCH = {"c2_0.6b_f16": 64, "c3_0.6b_q8": 64}
# the reference's default CPU thread count (src/ggml_graph.cpp:47)
REF_DEFAULT_THREADS = 8
SR = 16000
L2_FLUSH_BYTES = 256 << 20


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return pk, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(config):
    """Per-launch DRAM traffic of the dominant kernel for this workload, from
    the ncu figures committed in profiles/roofline_traffic.json, else None."""
    path = os.path.join(REPO, "profiles", "roofline_traffic.json")
    try:
        with open(path) as f:
            ent = json.load(f).get(config)
        return float(ent["bytes_per_launch"]) if ent else None
    except (OSError, ValueError, KeyError, TypeError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = f"/tmp/pkc_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        sm.append(float(parts[1]))
                        mx = float(parts[2])
                    except ValueError:
                        continue
                    for n, v in zip(names, parts[5:9]):
                        if v.lower() == "active":
                            reasons.add(n)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def workload(config, batch=None):
    """The global batch of a workload: every rank draws the same clips."""
    import synth
    b, lo, hi = synth.BATCHES[config]
    b = batch or GLOBAL_BATCH.get(config, b)
    pcm = synth.synth_batch(config, seed=1000, batch=b)
    return pcm, {"batch": b, "len_s": [lo, hi]}


def my_share(pcm, world, rank):
    """Indices of the clips this rank encodes: the library's LPT plan over
    the ranks (pkc_shard_plan, cost T'(1 + T'/8192) per clip)."""
    if world <= 1:
        return list(range(len(pcm)))
    import pkc
    assign = pkc.shard_plan([len(p) for p in pcm], world)
    return [i for i, a in enumerate(assign) if a == rank]


def combine_ranks(ms, e2e_ms, audio_s, wall_ms, world, device):
    """Whole-job timing: the slowest rank's times (MAX) and every rank's audio
    (SUM); on one rank the values pass through."""
    if world <= 1:
        return ms, e2e_ms, audio_s, wall_ms
    import torch
    import torch.distributed as dist
    vals = torch.tensor([ms, e2e_ms, audio_s, wall_ms], dtype=torch.float64, device=device)
    mx = vals.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    tot = vals.clone()
    dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    return mx[0].item(), mx[1].item(), tot[2].item(), mx[3].item()


# ----------------------------------------------------------------------- ours

def measure_encoder(model, pcm, dev, steps, warmup, world, profile=True):
    """One rank's share of the workload: device-resident steps (CUDA events
    per step, L2 flushed between steps outside the events), the per-kernel
    profile pass, and e2e steps through the host-buffer API. Returns the
    rank's figures (ms for `steps` steps)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import pkc
    n = [len(p) for p in pcm]
    res = {"audio_s": sum(n) / SR, "clips": len(pcm), "ms": 0.0, "e2e_ms": 0.0, "e2e_wall_ms": 0.0,
           "stats": [], "prof_steps": 0, "h2d": int(sum(n) * 4), "d2h": 0}
    d = model.info.d_model
    out_floats = int(sum(model.encoder_frames(model.mel_frames(x)) for x in n) * d) if n else 0
    res["d2h"] = out_floats * 4
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    if n:
        flat = np.concatenate(pcm).astype(np.float32)
        d_pcm = torch.from_numpy(flat).to(dev)
        d_out = torch.empty(out_floats, dtype=torch.float32, device=dev)

        def step():
            model.encode_pcm_device(d_pcm.data_ptr(), n, d_out.data_ptr(), stream=stream.cuda_stream)
    else:
        def step():
            pass
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    if n:
        model.encode_pcm_device(d_pcm.data_ptr(), n, d_out.data_ptr(), stream=stream.cuda_stream, sync=True)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    res["ms"] = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    if n:
        # the device path reports kernel errors through its error word on sync
        model.encode_pcm_device(d_pcm.data_ptr(), n, d_out.data_ptr(), stream=stream.cuda_stream, sync=True)
        # kernel launches of one timed step: the kernel nodes of its CUDA graph
        res["graph_kernels"] = model.last_graph_kernels(0)
    if profile and n:
        res["prof_steps"] = max(1, min(steps, 5))
        model.profile_enable(True)
        for _ in range(res["prof_steps"]):
            step()
        torch.cuda.synchronize(dev)
        res["stats"] = model.profile_read()
        model.profile_enable(False)
    # e2e: public host-buffer API, pinned PCM in, output to a pinned host buffer
    if n:
        host_pcm = [torch.from_numpy(p).pin_memory().numpy() for p in pcm]
        host_out = torch.empty(model.out_floats(n), dtype=torch.float32).pin_memory().numpy()
        for _ in range(max(1, warmup)):
            model.encode_pcm_batch(host_pcm, layout=pkc.LAYOUT_TIME_MAJOR, out=host_out)
        lib_stream = torch.cuda.ExternalStream(model.stream(), device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    if n:
        e0.record(lib_stream)
        for _ in range(steps):
            model.encode_pcm_batch(host_pcm, layout=pkc.LAYOUT_TIME_MAJOR, out=host_out)
        e1.record(lib_stream)
    torch.cuda.synchronize(dev)
    res["e2e_wall_ms"] = (time.perf_counter() - t0) * 1e3
    if n:
        res["e2e_ms"] = e0.elapsed_time(e1)
        res["host_pcm"] = host_pcm
    return res


def kernel_table(stats, prof_steps, peak, hbm):
    kernels = []
    tot_ms = sum(s["total_ms"] for s in stats) or 1.0
    for s in sorted(stats, key=lambda s: -s["total_ms"]):
        k = {"name": s["name"], "launches_per_step": s["launches"] / prof_steps,
             "ms_per_step": round(s["total_ms"] / prof_steps, 4), "share": round(s["total_ms"] / tot_ms, 4)}
        if s["flops"] > 0 and s["name"].startswith(("gemm", "attention")):
            k["tflops"] = round(s["flops"] / (s["total_ms"] / 1e3) / 1e12, 1)
            k["frac_tensor_peak"] = round(k["tflops"] / peak, 3)
        elif s["bytes"] > 0:
            k["gbs"] = round(s["bytes"] / (s["total_ms"] / 1e3) / 1e9, 1)
            k["frac_hbm_peak"] = round(k["gbs"] / hbm, 3)
        kernels.append(k)
    return kernels


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import pkc
    import synth

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = synth.CONFIGS[args.config]
    if rank == 0 or world == 1:
        path = synth.ensure_gguf(cfg)
    if world > 1:
        dist.barrier()
    path = synth.ensure_gguf(cfg)

    pcm_all, winfo = workload(args.config, args.batch)
    mine = my_share(pcm_all, world, rank)
    pcm = [pcm_all[i] for i in mine]

    t_open = time.perf_counter()
    model = pkc.Model(path, devices=(local_rank,))
    load = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in model.load_stats().items()}
    load["open_s"] = round(time.perf_counter() - t_open, 3)
    load["api"] = ("pkc_model_open: host re-pack once (or the PKC_PACK_CACHE pre-pack file), "
                   "page-locked image, concurrent per-device upload")
    d = model.info.d_model

    with ClockSampler(local_rank) as clk:
        r = measure_encoder(model, pcm, dev, args.steps, args.warmup, world)
    stats, prof_steps = r["stats"], max(1, r["prof_steps"])
    host_pcm = r.get("host_pcm", [])

    # ---- greedy transducer transcription (TDT / RNN-T models): PCM -> tokens
    # through pkc_transducer_greedy_pcm_batch, everything on the GPU (rank 0's share)
    trd = None
    if model.transducer_kind() > 0 and host_pcm and rank == 0:
        for _ in range(max(1, args.warmup)):
            model.transducer_greedy_pcm_batch(host_pcm)
        lib_stream = torch.cuda.ExternalStream(model.stream(), device=dev)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t_start.record(lib_stream)
        for _ in range(args.steps):
            toks = model.transducer_greedy_pcm_batch(host_pcm)
        t_end.record(lib_stream)
        torch.cuda.synchronize(dev)
        trd_ms = t_start.elapsed_time(t_end) / args.steps
        model.profile_enable(True)
        model.transducer_greedy_pcm_batch(host_pcm)
        torch.cuda.synchronize(dev)
        tst = {s["name"]: s["total_ms"] for s in model.profile_read()}
        model.profile_enable(False)
        trd = {"metric": "greedy " + ("TDT" if model.transducer_kind() == 2 else "RNN-T") +
                         " transcription RTFx (PCM -> tokens, encoder and decode on the GPU; rank 0's share)",
               "value": round(r["audio_s"] / (trd_ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(trd_ms, 3),
               "decode_ms": round(tst.get("transducer_decode", 0.0), 3),
               "joint_enc_gemm_ms": round(tst.get("gemm_joint_enc", 0.0), 4),
               "tokens_per_step": sum(len(t) for t in toks),
               "api": "pkc_transducer_greedy_pcm_batch (host buffers)"}

    # ---- CTC transcription (hybrid / CTC models): PCM -> tokens through
    # pkc_ctc_greedy_pcm_batch, host buffers (rank 0's share)
    ctc = None
    if model.ctc_classes() > 0 and host_pcm and rank == 0:
        for _ in range(max(1, args.warmup)):
            model.ctc_greedy_pcm_batch(host_pcm)
        lib_stream = torch.cuda.ExternalStream(model.stream(), device=dev)
        c_start = torch.cuda.Event(enable_timing=True)
        c_end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        c_start.record(lib_stream)
        for _ in range(args.steps):
            model.ctc_greedy_pcm_batch(host_pcm)
        c_end.record(lib_stream)
        torch.cuda.synchronize(dev)
        ctc_ms = c_start.elapsed_time(c_end) / args.steps
        model.profile_enable(True)
        model.ctc_greedy_pcm_batch(host_pcm)
        torch.cuda.synchronize(dev)
        cst = [s for s in model.profile_read() if s["name"].startswith(("ctc_", "gemm_ctc"))]
        model.profile_enable(False)
        ctc = {"metric": "CTC transcription RTFx (PCM -> tokens: encoder + CTC head on the GPU, greedy fold on "
                         "the host; rank 0's share)",
               "value": round(r["audio_s"] / (ctc_ms / 1e3), 1), "unit": UNIT, "ms_per_step": round(ctc_ms, 3),
               "classes": model.ctc_classes(), "api": "pkc_ctc_greedy_pcm_batch (host buffers)",
               "head_kernels": [{"name": s["name"], "ms": round(s["total_ms"], 4),
                                 **({"tflops": round(s["flops"] / (s["total_ms"] / 1e3) / 1e12, 1)} if s["flops"] > 0 else
                                    {"gbs": round(s["bytes"] / (s["total_ms"] / 1e3) / 1e9, 1)})} for s in cst]}
    model.close()

    ms_max, e2e_max, _, wall_max = combine_ranks(r["ms"], r["e2e_ms"], r["audio_s"], r["e2e_wall_ms"], world, dev)
    audio_total = sum(len(p) for p in pcm_all) / SR

    # ---- the q8_0 model of configuration 3 on the same global batch
    c3 = None
    if args.config == DEFAULT_CONFIG and not args.no_q8:
        c3 = measure_other("c3_0.6b_q8", pcm_all, mine, dev, args, rank, world)

    # ---- in-process multi-device path (pkc_model_open with all N devices,
    # pkc_encode_pcm_batch sharding the global batch across them): rank 0
    # alone, the other ranks waiting on a host-side barrier
    multi = None
    if world > 1 and not args.no_multi:
        multi = measure_multi_device(path, pcm_all, world, rank, args)

    if rank != 0:
        return None
    value = audio_total * args.steps / (ms_max / 1e3)
    peaks, peak_src = load_peaks()
    peak = peaks.get("bf16_tflops")
    peak_sus = peaks.get("bf16_tflops_sustained")
    hbm = peaks["hbm_gbs"]
    kernels = kernel_table(stats, prof_steps, peak, hbm)
    # roofline: the dominant kernel class (largest share of the profiled step)
    gemm = [s for s in stats if s["name"].startswith("gemm_")]
    dom = max(gemm, key=lambda s: s["total_ms"]) if gemm else None
    achieved = dom["flops"] / (dom["total_ms"] / 1e3) / 1e12 if dom else 0.0
    g_ms = sum(s["total_ms"] for s in gemm)
    g_fl = sum(s["flops"] for s in gemm)
    launches_per_step = sum(s["launches"] for s in stats) / prof_steps
    step_flops = sum(s["flops"] for s in stats) / prof_steps
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f16" if "bf16" not in args.config else "bf16",
        "data": "synthetic (seeded sines + noise; random-init weights, BASELINE.json init)",
        "config": {"workload": f"{args.config}: {cfg.n_layers}-layer d{d} FastConformer encoder "
                               f"({cfg.dtype} weights), PCM -> encoder output, global batch {winfo['batch']} clips "
                               f"of U({winfo['len_s'][0]},{winfo['len_s'][1]}) s sharded by utterance over "
                               f"{world} GPU(s)",
                   "global_batch": winfo["batch"], "audio_s_per_step": round(audio_total, 2),
                   "clips_on_rank0": len(pcm), "parallelism": f"utterance-sharded dp{world} (LPT, pkc_shard_plan)",
                   "l2": "256 MiB written between timed steps (L2 flush); per-step working set > 1 GB"},
        "e2e": {"value": round(audio_total * args.steps / (e2e_max / 1e3), 1), "unit": UNIT,
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                "api": "pkc_encode_pcm_batch (host buffers: pinned PCM in, pinned output buffer reused per step)",
                "wall_value": round(audio_total * args.steps / (wall_max / 1e3), 1),
                "note": "h2d / d2h bytes are rank 0's share"},
        "gpu_launches": int((r.get("graph_kernels") or round(launches_per_step)) * args.steps),
        "roofline": {"bound": "tensor", "kernel": f"{dom['name'] if dom else '-'} (tcgen05 GEMM class with the "
                                                  "largest share of the step)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3) if peak else None,
                     "frac_of_sustained": round(achieved / peak_sus, 3) if peak_sus else None,
                     "traffic": profile_traffic(args.config),
                     "launches_per_step": (dom["launches"] / prof_steps) if dom else 0,
                     "all_gemm_tflops": round(g_fl / (g_ms / 1e3) / 1e12, 1) if g_ms else None,
                     "step_tflops": round(step_flops / (ms_max / args.steps / 1e3) / 1e12, 1) if world == 1 else None,
                     "peak_source": f"{peak_src} bf16_tflops (burst dense f16/bf16 tensor peak); "
                                    f"frac_of_sustained against bf16_tflops_sustained"},
        "kernels": kernels,
        "clocks": clk.summary(),
    }
    line["load"] = load
    if c3 is not None:
        line["c3_q8"] = c3
    if multi is not None:
        line["multi_device_in_process"] = multi
    if ctc is not None:
        line["ctc"] = ctc
    if trd is not None:
        line["transducer"] = trd
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, path, pcm_all)
    return line


def measure_other(config, pcm_all, mine, dev, args, rank, world):
    """Device-resident and e2e throughput of another model on the same global
    batch and shard (the configuration-3 q8_0 weights)."""
    import torch.distributed as dist
    import pkc
    import synth
    if rank == 0 or world == 1:
        synth.ensure_gguf(synth.CONFIGS[config])
    if world > 1:
        dist.barrier()
    path = synth.ensure_gguf(synth.CONFIGS[config])
    model = pkc.Model(path, devices=(dev.index,))
    pcm = [pcm_all[i] for i in mine]
    r = measure_encoder(model, pcm, dev, args.steps, args.warmup, world, profile=(rank == 0))
    model.close()
    ms_max, e2e_max, _, _ = combine_ranks(r["ms"], r["e2e_ms"], r["audio_s"], r["e2e_wall_ms"], world, dev)
    audio_total = sum(len(p) for p in pcm_all) / SR
    if rank != 0:
        return None
    peaks, _ = load_peaks()
    cfg = synth.CONFIGS[config]
    prof_steps = max(1, r["prof_steps"])
    gemm = [s for s in r["stats"] if s["name"].startswith("gemm_")]
    g_ms = sum(s["total_ms"] for s in gemm)
    return {"workload": f"{config}: {cfg.n_layers}-layer d{cfg.d_model}, {cfg.dtype} weights dequantised inside "
                        f"the GEMM, the same global batch and shard",
            "value": round(audio_total * args.steps / (ms_max / 1e3), 1), "unit": UNIT,
            "ms_per_step": round(ms_max / args.steps, 3),
            "e2e": {"value": round(audio_total * args.steps / (e2e_max / 1e3), 1), "unit": UNIT,
                    "api": "pkc_encode_pcm_batch (host buffers)"},
            "all_gemm_tflops": round(sum(s["flops"] for s in gemm) / (g_ms / 1e3) / 1e12, 1) if g_ms else None,
            "kernels": kernel_table(r["stats"], prof_steps, peaks.get("bf16_tflops"), peaks["hbm_gbs"])[:8]}


def measure_multi_device(path, pcm_all, world, rank, args):
    """Rank 0 opens the model on all `world` GPUs in one process and encodes
    the global batch through pkc_encode_pcm_batch (LPT over the devices, one
    host thread per device); the other ranks have closed their models and
    wait on a gloo barrier (host-side, so their GPUs stay idle). Time: CUDA
    events on every device's library stream, the max over devices."""
    import torch
    import torch.distributed as dist
    import pkc
    g = dist.new_group(backend="gloo")
    out = None
    if rank == 0:
        model = pkc.Model(path, devices=tuple(range(world)))
        try:
            host_pcm = [torch.from_numpy(p).pin_memory().numpy() for p in pcm_all]
            host_out = torch.empty(model.out_floats([len(p) for p in pcm_all]),
                                   dtype=torch.float32).pin_memory().numpy()
            for _ in range(max(1, args.warmup)):
                model.encode_pcm_batch(host_pcm, layout=pkc.LAYOUT_TIME_MAJOR, out=host_out)
            evs = []
            for k in range(world):
                s = torch.cuda.ExternalStream(model.stream(k), device=torch.device("cuda", k))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                evs.append((s, a, b))
            for k in range(world):
                torch.cuda.synchronize(k)
            t0 = time.perf_counter()
            for s, a, _ in evs:
                a.record(s)
            for _ in range(args.steps):
                model.encode_pcm_batch(host_pcm, layout=pkc.LAYOUT_TIME_MAJOR, out=host_out)
            for s, _, b in evs:
                b.record(s)
            for k in range(world):
                torch.cuda.synchronize(k)
            wall = time.perf_counter() - t0
            ms = max(a.elapsed_time(b) for _, a, b in evs)
        finally:
            model.close()
        audio = sum(len(p) for p in pcm_all) / SR
        out = {"value": round(audio * args.steps / (ms / 1e3), 1), "unit": UNIT, "devices": world,
               "ms_per_step": round(ms / args.steps, 3), "wall_value": round(audio * args.steps / wall, 1),
               "api": "pkc_model_open(path, [0..N-1]) + pkc_encode_pcm_batch (host buffers, in-process LPT "
                      "sharding, one host thread per device)",
               "timing": "CUDA events on each device's library stream, max over devices"}
    dist.barrier(group=g)
    return out


# ----------------------------------------------------------------------- CPU

def cpu_sample(pcm_all, k=4):
    """A bounded sample of the workload that keeps its length mix: k clips of
    the batch at evenly spaced length quantiles (for U(2, 35) s clips about
    1/8, 3/8, 5/8 and 7/8 of the way through the sorted lengths)."""
    order = sorted(range(len(pcm_all)), key=lambda i: len(pcm_all[i]))
    n = len(order)
    picks = sorted({order[min(n - 1, int((2 * q + 1) * n / (2 * k)))] for q in range(k)})
    return [pcm_all[i] for i in picks]


def cpu_threads():
    """BLAS threads numpy uses (all host cores unless limited)."""
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        n = max((d.get("num_threads", 0) for d in info if d.get("user_api") == "blas"), default=0)
        if n:
            return n
    except Exception:
        pass
    return os.cpu_count()


def cpu_encode(w, clip):
    """The reference's CPU path on one clip: parakeet.cpp's own MelFrontend
    (compiled from its sources, oracle/_ref) when present, then the encoder
    restatement in float32 with every BLAS thread."""
    import numpy as np
    import oracle
    import ref
    if ref.available():
        feats = ref.mel(clip, n_mels=w.n_mels, n_fft=w.n_fft, hop=w.hop, win_length=len(w.t["preprocessor.featurizer.window"]),
                        preemph=w.preemph, mag_power=w.mag_power, log_guard=w.log_guard,
                        per_feature=w.per_feature, window=w.t["preprocessor.featurizer.window"].astype(np.float32),
                        fb=w.fb())
    else:
        feats = oracle.mel_frontend(w, clip)
    with oracle.compute_dtype(np.float32):
        return oracle.encoder_forward_batch(w, feats[None], [feats.shape[1]])


def cpu_sample_desc(sample, reps):
    secs = [round(len(c) / SR, 1) for c in sample]
    return (f"{reps} pass(es) over {len(sample)} clips of the batch at its length quantiles ({secs} s); "
            f"encoder = numpy float32 restatement of the reference's graph ({cpu_threads()} BLAS threads; the "
            f"reference's ggml CPU default is {REF_DEFAULT_THREADS} threads), mel = parakeet.cpp MelFrontend "
            f"(oracle/_ref); parakeet.cpp's ggml encoder itself is not buildable here (ggml absent)")


def cpu_baseline(args, path, pcm_all):
    import oracle
    w = oracle.Weights(path)
    sample = cpu_sample(pcm_all)
    audio = sum(len(c) for c in sample) / SR
    cpu_encode(w, sample[0])  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        for c in sample:
            cpu_encode(w, c)
        reps += 1
        if time.perf_counter() - t0 > 10.0 or reps >= 3:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(audio / dt, 3), "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": cpu_sample_desc(sample, reps)}


# ----------------------------------------------------------------- streaming

def stream_windows(sch, T):
    """The model's chunk schedule over T mel frames: (lo, hi, is_last)."""
    out, idx, first = [], 0, True
    while idx < T:
        size = sch["chunk_size_first"] if first else sch["chunk_size"]
        hi = min(idx + size, T)
        lo = idx if first else max(0, idx - sch["pre_encode_cache_size"])
        out.append((lo, hi, hi >= T))
        idx += size
        first = False
    return out


def stream_launches(cfg, n_windows, n_tc_changes):
    """Kernels of one stream (16-bit weights): per chunk 6 subsampling
    launches, 11 per layer (the pre-norms run inside their skinny GEMMs; the
    layer's output norm is its own kernel), the cache roll and the cache-fill
    update; the positional table and every layer's linear_pos (2) when the
    chunk length changes."""
    return n_windows * (6 + 11 * cfg.n_layers + 2) + 2 * n_tc_changes


def run_stream(args, rank, world, local_rank):
    """Cache-aware streaming encoder (pkc_stream_*): one stream of
    args.stream_seconds of synthetic log-mel per GPU, fed window by window.
    A step is the whole stream; value = audio seconds / device seconds."""
    import numpy as np
    import torch
    import pkc
    import synth
    if world > 1:
        raise SystemExit("the streaming bench runs on one GPU (one stream per process)")
    cfg = synth.STREAM_CONFIGS[args.config]
    path = synth.ensure_gguf(cfg)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    model = pkc.Model(path, devices=(local_rank,))
    sch = model.stream_schedule()
    d = model.info.d_model
    seconds = args.stream_seconds
    T = int(round(seconds * SR / cfg.hop_length))
    mel = np.random.default_rng(7).standard_normal((cfg.n_mels, T)).astype(np.float32)
    wins = stream_windows(sch, T)
    win_mel = [np.ascontiguousarray(mel[:, lo:hi]) for lo, hi, _ in wins]
    s = pkc.Stream(model)
    ext = torch.cuda.ExternalStream(model.stream(0), device=dev)

    def one_stream(lat=None):
        s.reset()
        frames = 0
        for (lo, hi, last), wm in zip(wins, win_mel):
            t = time.perf_counter()
            o = s.step(wm, last)
            if lat is not None:
                lat.append((time.perf_counter() - t) * 1e3)
            frames += o.shape[0]
        return frames

    for _ in range(args.warmup):
        frames = one_stream()
    lat = []
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clk:
        t0 = time.perf_counter()
        ev0.record(ext)
        for _ in range(args.steps):
            one_stream(lat)
        ev1.record(ext)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
    dev_ms = ev0.elapsed_time(ev1)
    s.close()
    audio = seconds * args.steps
    lat = sorted(lat)
    pct = lambda q: round(lat[min(len(lat) - 1, int(q * len(lat)))], 3)
    # roofline: one chunk reads every encoder weight once (f16: 2 bytes a parameter)
    n_params = sum(int(np.prod(a.shape)) for n, a in synth.model_tensors(cfg) if n.startswith("encoder."))
    wbytes = 2 * n_params
    per_chunk_s = dev_ms / 1e3 / (args.steps * len(wins))
    peaks, peak_src = load_peaks()
    hbm = peaks.get("hbm_gbs")
    achieved = wbytes / per_chunk_s / 1e9
    n_tc = 2 if len(wins) > 1 else 1
    line = {
        "metric": "cache-aware streaming encoder RTFx (audio-s/s of one stream) and per-chunk latency",
        "value": round(audio / (dev_ms / 1e3), 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": cfg.dtype if cfg.dtype in ("f16", "bf16") else "f16",
        "data": "synthetic log-mel (seeded N(0,1) features), random-init weights of the model class",
        "config": {"workload": f"{args.config}: {cfg.n_layers}-layer d{d} causal FastConformer, one stream of "
                               f"{seconds:g} s ({T} mel frames) in {len(wins)} windows "
                               f"({sch['chunk_size_first']}, then {sch['pre_encode_cache_size']} + {sch['chunk_size']} mel frames)",
                   "schedule": sch, "l2": "weights (2 bytes x {:.0f} M) exceed L2; no flush".format(n_params / 1e6)},
        "chunk_latency_ms": {"p50": pct(0.5), "p90": pct(0.9), "p99": pct(0.99), "max": round(lat[-1], 3),
                             "chunks": len(lat), "audio_ms_per_chunk": round(1e3 * sch["chunk_size"] * cfg.hop_length / SR, 1),
                             "api": "pkc_stream_step (host mel window in, host frames out, synchronous)"},
        "e2e": {"value": round(audio / wall, 1), "unit": UNIT,
                "h2d_bytes_per_step": int(sum(w.nbytes for w in win_mel)),
                "d2h_bytes_per_step": int(frames * d * 4), "api": "pkc_stream_step"},
        "gpu_launches": int(stream_launches(cfg, len(wins), n_tc) * args.steps),
        "roofline": {"bound": "hbm", "kernel": "one chunk through every layer (each weight read once)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 3) if hbm else None, "traffic": None,
                     "peak_source": f"{peak_src} hbm_gbs",
                     "note": "latency-bound: a chunk is 2 frames, so its cost is launches and dependent "
                             "small GEMMs, not bytes"},
        "clocks": clk.summary(),
    }
    # serving form: args.stream_batch streams stepped together (pkc_stream_step_batch)
    S = args.stream_batch
    if S > 1:
        streams = [pkc.Stream(model) for _ in range(S)]
        mels_b = [np.random.default_rng(100 + i).standard_normal((cfg.n_mels, T)).astype(np.float32) for i in range(S)]
        win_b = [[np.ascontiguousarray(mb[:, lo:hi]) for lo, hi, _ in wins] for mb in mels_b]

        def batch_stream(lat=None):
            for s in streams:
                s.reset()
            for k, (lo, hi, last) in enumerate(wins):
                t = time.perf_counter()
                pkc.stream_step_batch(streams, [wb[k] for wb in win_b], [last] * S)
                if lat is not None:
                    lat.append((time.perf_counter() - t) * 1e3)

        for _ in range(args.warmup):
            batch_stream()
        blat = []
        torch.cuda.synchronize(dev)
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(ext)
        tb = time.perf_counter()
        for _ in range(args.steps):
            batch_stream(blat)
        b1.record(ext)
        torch.cuda.synchronize(dev)
        bwall = time.perf_counter() - tb
        bms = b0.elapsed_time(b1)
        for s in streams:
            s.close()
        blat = sorted(blat)
        bp = lambda q: round(blat[min(len(blat) - 1, int(q * len(blat)))], 3)
        line["batched"] = {"streams": S, "value": round(S * audio / (bms / 1e3), 1), "unit": UNIT,
                           "e2e_value": round(S * audio / bwall, 1),
                           "chunk_latency_ms": {"p50": bp(0.5), "p99": bp(0.99), "max": round(blat[-1], 3)},
                           "api": "pkc_stream_step_batch (all streams' windows in one chunk step)"}
    if not args.no_cpu_baseline:
        import oracle
        w = oracle.Weights(path)
        enc = oracle.StreamingEncoder(w)
        n_cpu = min(len(wins), 8)
        t0 = time.perf_counter()
        for (lo, hi, last), wm in list(zip(wins, win_mel))[:n_cpu]:
            enc.step(wm, False)
        dt = time.perf_counter() - t0
        audio_cpu = n_cpu * sch["chunk_size"] * cfg.hop_length / SR
        line["cpu_baseline"] = {"value": round(audio_cpu / dt, 3), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                                "sample": f"the first {n_cpu} windows of the stream through the numpy float64 "
                                          "restatement of StreamingEncoder::step"}
    model.close()
    return line


def run_reference_stream(args):
    """Reference arm of the streaming configurations: the numpy float64
    restatement of StreamingEncoder::step (ggml absent, so the reference's own
    streaming graph cannot run here), a bounded prefix of the same stream."""
    import numpy as np
    import oracle
    import synth
    cfg = synth.STREAM_CONFIGS[args.config]
    path = synth.ensure_gguf(cfg)
    w = oracle.Weights(path)
    sc = oracle.StreamCfg(w)
    T = int(round(args.stream_seconds * SR / cfg.hop_length))
    mel = np.random.default_rng(7).standard_normal((cfg.n_mels, T)).astype(np.float32)
    wins = oracle.stream_schedule(sc, T)[:8]
    audio = len(wins) * sc.chunk_main * cfg.hop_length / SR
    enc = oracle.StreamingEncoder(w)
    for _ in range(args.warmup):
        enc.reset()
        for lo, hi, last in wins:
            enc.step(mel[:, lo:hi], False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        enc.reset()
        for lo, hi, last in wins:
            enc.step(mel[:, lo:hi], False)
    dt = time.perf_counter() - t0
    v = audio * args.steps / dt
    return {"metric": "cache-aware streaming encoder RTFx (audio-s/s of one stream) and per-chunk latency",
            "value": round(v, 3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "impl": "reference", "data": "synthetic",
            "config": {"workload": f"{args.config} (bounded CPU sample)", "sample": f"first {len(wins)} windows per step"},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": f"first {len(wins)} windows of the stream per step; numpy float64 restatement"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference(args, rank, world):
    """The reference arm: parakeet.cpp's CPU path on the host cores (rank 0
    alone; other ranks exit without work). Each step encodes the next clip of
    the length-quantile sample of the same global batch."""
    if rank != 0:
        return None
    import oracle
    import synth
    if args.config in synth.STREAM_CONFIGS:
        return run_reference_stream(args)
    cfg = synth.CONFIGS[args.config]
    path = synth.ensure_gguf(cfg)
    pcm_all, winfo = workload(args.config, args.batch)
    w = oracle.Weights(path)
    sample = cpu_sample(pcm_all)
    for k in range(args.warmup):
        cpu_encode(w, sample[k % len(sample)])
    audio = 0.0
    t0 = time.perf_counter()
    for k in range(args.steps):
        c = sample[k % len(sample)]
        cpu_encode(w, c)
        audio += len(c) / SR
    dt = time.perf_counter() - t0
    v = audio / dt
    desc = cpu_sample_desc(sample, 1).replace("1 pass(es) over", f"{args.steps} steps cycling through")
    return {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic",
            "config": {"workload": f"{args.config}: global batch {winfo['batch']} clips of "
                                   f"U({winfo['len_s'][0]},{winfo['len_s'][1]}) s (bounded CPU sample: one clip per step)",
                       "sample": desc},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=DEFAULT_CONFIG)
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-q8", action="store_true", help="skip the configuration-3 q8_0 measurement")
    ap.add_argument("--no-multi", action="store_true", help="skip the in-process multi-device measurement")
    ap.add_argument("--stream-seconds", type=float, default=20.0,
                    help="audio per stream for the streaming configurations")
    ap.add_argument("--stream-batch", type=int, default=32,
                    help="streams stepped together in the streaming configurations' batched measurement")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        import synth
        if args.config in synth.STREAM_CONFIGS:
            line = run_stream(args, rank, world, local_rank)
        else:
            line = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
