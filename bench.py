"""Throughput of OmniVoice's generator hot path on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c2|c1|c3|c5|c4|codec|encode|longtext]
                  [--noise device|reference]

A "step" is one full 32-step CFG unmasking generation of the workload.
The default workload is BASELINE config 2 (120 text tokens + 250 masked
frames = one 10 s utterance) on every GPU: independent utterances are
replicated across ranks with no collective on the data path (weak
scaling).  `--workload c4` runs the batched config (64 utterances,
partitioned across ranks by longest-processing-time, strong scaling).
`--workload codec` times the audio tokenizer's decoder instead (codes of a
250-frame chunk to 24 kHz audio, replicas only); `--workload encode` the
encoder (a 6 s reference voice to codes, replicas only); `--workload longtext` a
60 s text as four chunks, generated (chunk 0, then chunks 1-3 batched) and
decoded, beside the reference's chunk-by-chunk order.

value: audio seconds generated per second, whole job, inputs resident in
HBM, device time (CUDA events on the generator's stream, max over ranks).
e2e:   the same metric through the C-ABI with host buffers (upload of the
inputs and download of the codes inside the timed region), wall clock.
Rank 0 prints one JSON line.  `--impl reference` times the CPU restatement
of the reference generator (oracle/, the reference's own generator is HIP
code that cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "audio-sec generated per sec (32-step CFG) at 1/2/4/8 B200; per-step backbone ms"
FRAME_RATE = 25.0
VOCAB = 151936


# ------------------------------------------------------------- workloads

def _input(rng, text, ref_frames, target):
    from omnivoice_b200 import ConditionalInput
    text_ids = rng.integers(0, VOCAB, size=text).tolist()
    ref = rng.integers(0, 1024, size=(8, ref_frames)).astype(np.int32) if ref_frames else None
    return ConditionalInput.build(text_ids, ref, target)


WORKLOADS = {
    "c1": ("config1: 40 text + 100 masked frames (4 s), 32-step CFG", 0, [(40, 0, 100)]),
    "c2": ("config2: 120 text + 250 masked frames (10 s), 32-step CFG", 1, [(120, 0, 250)]),
    "c3": ("config3: 180 text + 150 reference + 375 masked frames (15 s), 32-step CFG", 2,
           [(180, 150, 375)]),
    "c5": ("config5: 300 text + 375 reference + 750 masked frames (30 s), 32-step CFG", 3,
           [(300, 375, 750)]),
}


def batched_set(seed=4, count=64):
    """64 utterances, F ~ U[50, 750], text = round(0.4 F),
    half with 125-250 frames of reference codes."""
    rng = np.random.default_rng(seed)
    frames = rng.integers(50, 751, size=count)
    with_ref = set(rng.permutation(count)[: count // 2].tolist())
    specs = []
    for i, f in enumerate(frames):
        ref = int(rng.integers(125, 251)) if i in with_ref else 0
        specs.append((int(round(0.4 * f)), ref, int(f)))
    return rng, specs


def utterance_cost(text, ref, target):
    from omnivoice_b200.scheduler import utterance_cost as cost
    return cost(text + ref + target, target)


def lpt_partition(specs, ranks):
    """Longest-processing-time-first assignment of utterances to ranks
    (omnivoice_b200.scheduler, the same partition generate_data_parallel
    uses)."""
    from omnivoice_b200.scheduler import lpt_partition as lpt
    return lpt([utterance_cost(*s) for s in specs], ranks)


def make_workload(name, rank, world):
    if name == "c4":
        rng, specs = batched_set()
        inputs_all = [_input(rng, *s) for s in specs]
        parts, load = lpt_partition(specs, world)
        mine = parts[rank]
        desc = "config4: 64 utterances, F~U[50,750], LPT-partitioned across ranks"
        total_audio = sum(s[2] for s in specs) / FRAME_RATE
        seeds_all = [1000 + i for i in range(len(specs))]
        return (desc, [inputs_all[i] for i in mine], [seeds_all[i] for i in mine], total_audio,
                "strong", {"imbalance_max_over_mean": max(load) / (sum(load) / world),
                           "_all": (inputs_all, seeds_all)})
    desc, seed, specs = WORKLOADS[name]
    rng = np.random.default_rng(seed)
    inputs = [_input(rng, *s) for s in specs]
    total_audio = world * sum(s[2] for s in specs) / FRAME_RATE
    return desc, inputs, [seed + 100 * rank for _ in specs], total_audio, "weak", {}


# -------------------------------------------------------------- helpers

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during timing."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, value in zip(names, parts[2:]):
                if value.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# DRAM bytes per launch of each kernel class, from one ncu capture of the
# default workload (profiles/step_launches_config2.md: dram__bytes_read.sum +
# dram__bytes_write.sum per launch).
NCU_TRAFFIC = {
    ("c2", "gemm_gate_up_swiglu"): 13.89e6,
    ("c2", "gemm_down_residual"): 12.68e6,
    ("c2", "gemm_qkv_qknorm_rope"): 9.89e6,
    ("c2", "attention"): 5.15e6,
    ("c2", "gemm_o_residual"): 9.31e6,
}
TENSOR_CLASSES = ("gemm_qkv_qknorm_rope", "attention", "gemm_o_residual", "gemm_gate_up_swiglu",
                  "gemm_down_residual", "gemm_audio_head")


def roofline(prof, workload, clocks, gemm_flops, gemm_ms):
    """Roofline of the dominant kernel class of one profiled step: the class
    with the most device time (CUDA events around each launch of a captured
    step on the generator's stream).  achieved = its algorithmic FLOPs (or
    bytes) per launch / its average launch time.  peak = the measured cuBLAS
    bf16 GEMM rate (burst; the sustained figure when the run was power
    capped) or the measured copy bandwidth."""
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    capped = "sw_power_cap" in (clocks or {}).get("reasons", [])
    if peaks:
        tensor_peak = peaks.get("bf16_tflops_sustained" if capped else "bf16_tflops")
        hbm_peak, kind = peaks.get("hbm_gbs"), "measured" + (" (sustained)" if capped else " (burst)")
    else:
        tensor_peak, hbm_peak, kind = 1590.0, 6650.0, "fallback"
    top = max(prof, key=lambda k: k["ms"])
    launches = max(top["launches"], 1)
    per_launch_s = top["ms"] / 1e3 / launches
    if top["name"] in TENSOR_CLASSES:
        achieved = top["flops"] / launches / per_launch_s / 1e12
        bound, unit, peak = "tensor", "TFLOP/s", tensor_peak
    else:
        achieved = top["bytes"] / launches / per_launch_s / 1e9
        bound, unit, peak = "hbm", "GB/s", hbm_peak
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak if peak else None,
            "traffic": NCU_TRAFFIC.get((workload, top["name"])),
            "kernel": top["name"], "launches_per_step": top["launches"],
            "us_per_launch": per_launch_s * 1e6, "peak_kind": kind,
            "all_gemms_tflops": gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None}


def cpu_baseline(inputs, threads):
    """The oracle (CPU restatement of the reference generator) on one step
    of the workload's first utterance, extrapolated to 32 steps."""
    from oracle import binding
    binding.oracle().oc_set_threads(threads)
    cfg = binding.config()
    model = binding.OracleModel(cfg, 0)
    inp = inputs[0]
    t0 = time.perf_counter()
    logits = model.forward(inp.ids, inp.audio_start, inp.target_frames)
    pred, conf = binding.score(logits, inp.target_frames)
    codes = np.full((8, inp.target_frames), 1024, np.int32)
    binding.select(8 * inp.target_frames // 32, pred, conf, codes,
                   gumbel=binding.reference_gumbel(0, 8 * inp.target_frames))
    step_s = time.perf_counter() - t0
    model.close()
    audio = inp.target_frames / FRAME_RATE
    return {"value": audio / (32 * step_s), "unit": "audio_s/s", "cores": threads, "kind": "port",
            "sample": f"one forward+score+select step of the workload's first utterance "
                      f"({step_s:.2f} s), x32 extrapolated to the full generation"}


# ------------------------------------------------------------------ arms

def run_reference(args, rank, world):
    """--impl reference: the CPU restatement timed on the host cores.

    Each step is a bounded sample of one generation of the workload's first
    utterance: a forward with 0 layers (embedding + head) and one with 2
    layers are timed, with the scoring and the position choice; the full
    generation time is extrapolated as 32 x (t0 + 28 (t2 - t0) / 2 + t_tail)."""
    if rank != 0:
        return
    from oracle import binding
    threads = os.cpu_count() or 1
    binding.oracle().oc_set_threads(threads)
    desc, inputs, seeds, total_audio, scaling, extra = make_workload(args.workload, 0, 1)
    model = binding.OracleModel(binding.config(), 0)
    inp = inputs[0]
    F = inp.target_frames

    def one_step():
        s = time.perf_counter()
        model.forward(inp.ids, inp.audio_start, F, layers=0)
        t0 = time.perf_counter() - s
        s = time.perf_counter()
        logits = model.forward(inp.ids, inp.audio_start, F, layers=2)
        t2 = time.perf_counter() - s
        s = time.perf_counter()
        pred, conf = binding.score(logits, F)
        binding.select(8 * F // 32, pred, conf, np.full((8, F), 1024, np.int32),
                       gumbel=binding.reference_gumbel(0, 8 * F))
        t_tail = time.perf_counter() - s
        return 32 * (t0 + 28 * max(t2 - t0, 0.0) / 2 + t_tail)

    for _ in range(max(1, args.warmup)):
        one_step()
    gen_s = float(np.mean([one_step() for _ in range(args.steps)]))
    value = (F / FRAME_RATE) / gen_s
    line = {"metric": METRIC, "value": value, "unit": "audio_s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": gen_s * 1e3,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": desc + " (first utterance)",
                       "implementation": "oracle/: CPU restatement of the reference generator; "
                                         "the reference's generator is HIP-only"},
            "cpu_baseline": {"value": value, "unit": "audio_s/s", "cores": threads, "kind": "port",
                             "sample": "per step: forwards with 0 and 2 layers + score + select "
                                       "timed, extrapolated to 28 layers and 32 steps"},
            "e2e": {"value": value, "unit": "audio_s/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    model.close()
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank, dist):
    import torch

    from omnivoice_b200 import DecodingConfig, Generator
    from omnivoice_b200 import _native as N

    torch.cuda.set_device(local_rank)
    lib = N.lib()
    desc, inputs, seeds, total_audio, scaling, extra = make_workload(args.workload, rank, world)
    all_inputs = extra.pop("_all", None)
    dec = DecodingConfig()
    gen = Generator.synthetic(weight_seed=0, device=local_rank)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Device-resident timing: inputs uploaded once, K full generations.
    gen.prepare(inputs, dec, seeds, noise=args.noise)
    st = gen.stats()
    stream = st.stream
    for _ in range(args.warmup):
        gen.run()
    ev0, ev1 = ctypes.c_void_p(), ctypes.c_void_p()
    N.check(lib.ov_event_create(ctypes.byref(ev0)))
    N.check(lib.ov_event_create(ctypes.byref(ev1)))
    N.check(lib.ov_stream_sync(stream))
    gpu_index = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = gpu_index[local_rank] if len(gpu_index) > local_rank and gpu_index[0] else str(local_rank)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_index) as clocks:
        N.check(lib.ov_event_record(ev0, stream))
        for _ in range(args.steps):
            gen.run()
        N.check(lib.ov_event_record(ev1, stream))
        N.check(lib.ov_event_sync(ev1))
    ms = ctypes.c_float()
    N.check(lib.ov_event_elapsed_ms(ev0, ev1, ctypes.byref(ms)))
    torch.cuda.synchronize()
    barrier()
    t_max = max_over_ranks(ms.value)
    ms_per_gen = t_max / args.steps
    value = total_audio * args.steps / (t_max / 1e3)
    results = gen.fetch()
    assert all(((r.codes >= 0) & (r.codes < 1024)).all() for r in results)

    # Per-kernel-class device time of one step (CUDA events between the
    # kernels of a captured step, on the generator's stream).
    prof = gen.profile_step()
    st = gen.stats()
    # The profiled replay serialises the kernels (an event between each two,
    # so no programmatic-launch overlap): its sums are per-class shares.  The
    # per-step backbone time is the measured full step apportioned by the
    # share of everything but score and select.
    serial_ms = sum(k["ms"] for k in prof)
    backbone_serial_ms = sum(k["ms"] for k in prof if k["name"] not in ("score", "select"))
    backbone_ms = ms_per_gen / max(st.steps_run, 1) * backbone_serial_ms / max(serial_ms, 1e-9)
    gemms = [k for k in prof if k["name"].startswith("gemm")]
    gemm_ms = sum(k["ms"] for k in gemms)
    gemm_flops = sum(k["flops"] for k in gemms)

    # End to end through the public API with host buffers: the C-ABI batch
    # call per rank; for the batched workload the data-parallel scheduler
    # (partition on the host, gather of the codes to rank 0).
    def e2e_once():
        if all_inputs is None:
            gen.generate_batch(inputs, dec, seeds, noise=args.noise)
        else:
            from omnivoice_b200.scheduler import generate_data_parallel
            generate_data_parallel(all_inputs[0], dec, all_inputs[1],
                                   lambda b, d, s: gen.generate_batch(b, d, s, noise=args.noise))

    for _ in range(max(1, args.warmup // 2)):
        e2e_once()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_once()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    st_e2e = gen.stats()
    e2e_value = total_audio * args.steps / e2e_s

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline(inputs, os.cpu_count() or 1)
    gen.close()

    if rank != 0:
        return
    launches_per_gen = st.kernels_per_step * st.steps_run + st.kernels_per_reset
    line = {
        "metric": METRIC, "value": value, "unit": "audio_s/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_gen,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": desc, "rows_per_step": st.rows,
                   "steps_per_generation": st.steps_run,
                   "gflop_per_step": st.flops_per_step / 1e9, "noise": args.noise,
                   "weights": "random init N(0,0.02) (synthetic), fp16",
                   "l2_policy": "inputs larger than L2: every step streams 0.93 GB of weights",
                   "parallelism": f"dp{world} ({'replicas' if scaling == 'weak' else 'LPT partition'}), no collectives",
                   **extra},
        "backbone_ms_per_step": backbone_ms,
        "backbone_ms_serialised": backbone_serial_ms,
        "full_step_ms": ms_per_gen / max(st.steps_run, 1),
        "roofline": roofline(prof, args.workload, clocks.summary(), gemm_flops, gemm_ms),
        "cpu_baseline": base,
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_value, "unit": "audio_s/s",
                "h2d_bytes_per_step": st_e2e.h2d_bytes, "d2h_bytes_per_step": st_e2e.d2h_bytes,
                "timing": "wall clock around ov_generator_generate_batch"
                          + (" via omnivoice_b200.scheduler.generate_data_parallel"
                             if all_inputs is not None else "")},
        "gpu_launches": launches_per_gen * args.steps,
        "kernels": [{k["name"]: round(k["ms"], 4), "launches": k["launches"],
                     "tflops": round(k["flops"] / (k["ms"] / 1e3) / 1e12, 1) if k["flops"] and k["ms"] else None,
                     "gbs": round(k["bytes"] / (k["ms"] / 1e3) / 1e9, 1) if k["bytes"] and k["ms"] else None}
                    for k in prof],
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------- codec decoder (f1 row)

CODEC_FRAMES = 250  # one 10 s chunk, the generator's config-2 output


def codec_flops(cfg, frames):
    """Algorithmic float32 FLOPs of one decode (the reference's products,
    codec.cpp:215-253): fc2 after the codebook sum, every convolution as
    2 x rows x cout x cin x taps (a transposed one over its input rows)."""
    lat, hid = cfg.latent_channels, cfg.semantic_hidden + cfg.latent_channels
    total = 2 * frames * lat * hid
    rows, ch = frames, cfg.decoder_channels
    total += 2 * rows * ch * lat * 7
    for s in cfg.upsampling_ratios:
        out = ch // 2
        total += 2 * rows * (2 * s) * out * ch       # ConvTranspose1d, 2 s taps
        rows *= s
        total += 3 * (2 * rows * out * out * 7 + 2 * rows * out * out)
        ch = out
    return total + 2 * rows * ch * 7


def run_codec(args, rank, world):
    """--workload codec: the audio tokenizer's decoder (codes -> 24 kHz
    audio) on a 250-frame chunk; replicas only (each rank decodes its own
    chunk, no collective).  value: audio seconds decoded per second, codes
    and audio resident in HBM (CUDA events on the decode stream, max over
    ranks); e2e: through ov_codec_decode with host codes and host audio."""
    import torch

    from omnivoice_b200.codec import Codec, CodecConfig
    cfg = CodecConfig()
    codec = Codec.synthetic(cfg, seed=1)
    rng = np.random.default_rng(rank)
    codes_h = rng.integers(0, cfg.codebook_size, (cfg.codebooks, CODEC_FRAMES)).astype(np.int32)
    codes = torch.from_numpy(codes_h).cuda()
    audio = torch.empty(CODEC_FRAMES * cfg.frame_samples, device="cuda")
    # Inputs are 250 x 8 codes; the signals it writes (7.7 M samples x 32
    # channels x 4 planes in the last block) exceed L2, so no flush.
    stream = torch.cuda.Stream()
    for _ in range(max(3, args.warmup)):
        codec.decode_device(codes, audio, stream.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            codec.decode_device(codes, audio, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_audio = codec.decode(codes_h)
    e2e_s = (time.perf_counter() - t0) / args.steps
    assert np.isfinite(host_audio).all()
    seconds = CODEC_FRAMES / FRAME_RATE
    flops = codec_flops(cfg, CODEC_FRAMES)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tf32_peak = (peaks.get("bf16_tflops") or 1590.0) / 2
    line = {
        "metric": "audio-sec decoded per sec (codec decoder, 10 s chunk)",
        "value": world * seconds / (ms / 1e3), "unit": "audio_s/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (split tf32)",
        "data": "synthetic codes, random-init decoder weights",
        "config": {"workload": f"codec decode of {CODEC_FRAMES} frames (8 x 1024 codes) -> "
                               f"{CODEC_FRAMES * cfg.frame_samples} samples",
                   "parallelism": f"replicas{world}", "l2": "signals exceed L2, no flush"},
        "roofline": {"bound": "tensor", "achieved": 3 * flops / (ms / 1e3) / 1e12,
                     "peak": tf32_peak, "unit": "TFLOP/s",
                     "frac": 3 * flops / (ms / 1e3) / 1e12 / tf32_peak, "traffic": None,
                     "note": "tf32 MMA FLOPs (3 products per float32 product) over half the "
                             "measured bf16 peak (tf32 runs at half the f16 rate)"},
        "e2e": {"value": seconds / e2e_s, "unit": "audio_s/s",
                "h2d_bytes_per_step": int(codes_h.nbytes),
                "d2h_bytes_per_step": int(host_audio.nbytes)},
        "gpu_launches": args.steps * (3 + 7 * len(cfg.upsampling_ratios)),
        "clocks": clocks.summary(),
    }
    if not args.no_cpu_baseline:
        from oracle import codec as oc
        shape = oc.CodecShape()
        weights = oc.synthetic_weights(shape, 1)
        sample = rng.integers(0, 1024, (8, 3))
        t0 = time.perf_counter()
        oc.decode(weights, shape, sample)
        per_frame = (time.perf_counter() - t0) / 3
        line["cpu_baseline"] = {"value": 1 / FRAME_RATE / per_frame, "unit": "audio_s/s",
                                "cores": os.cpu_count(), "kind": "port",
                                "sample": "oracle/codec.py (numpy float64) decoding 3 frames, "
                                          "per-frame time scaled to the chunk"}
    if rank == 0:
        print(json.dumps(line), flush=True)


ENCODE_SECONDS = 6.0       # config 3's voice-clone prompt: a 6 s reference (150 frames)


def encoder_flops(cfg, samples: int) -> float:
    """Multiply-add FLOPs of one encode (codec_encoder.cpp:249-458) of
    `samples` 24 kHz samples with EncoderConfig `cfg`."""
    flops = 0.0
    n = int(np.ceil(samples * cfg.semantic_sample_rate / cfg.sample_rate)) + 320
    cin = 1
    for ch, k, st in zip(cfg.conv_channels, cfg.conv_kernels, cfg.conv_strides):
        n = (n - k) // st + 1
        flops += 2.0 * n * ch * cin * k
        cin = ch
    steps, h, i = n, cfg.hidden_size, cfg.intermediate_size
    flops += 2.0 * steps * cin * h + 2.0 * steps * h * (h // cfg.position_groups) * cfg.position_kernel
    flops += cfg.layers * (2.0 * steps * (4 * h * h + 2 * h * i) + 4.0 * steps * steps * h)
    frames = samples // cfg.frame_samples
    flops += 2.0 * frames * h * h * 25                     # semantic encoder: 25 taps of h x h
    t, ch = samples, cfg.encoder_channels
    flops += 2.0 * t * ch * 7
    for s in cfg.downsampling_ratios:
        flops += 3 * 2.0 * t * ch * ch * 8 + 2.0 * (t // s) * 2 * ch * ch * 2 * s
        t, ch = t // s, 2 * ch
    joint = h + cfg.latent_channels
    flops += 2.0 * frames * cfg.latent_channels * ch * 3 + 2.0 * frames * joint * joint
    flops += frames * cfg.codebooks * 4.0 * cfg.codebook_size * cfg.codebook_dim
    return flops


def run_encode(args, rank, world):
    """--workload encode: the audio tokenizer's encoder (voice cloning: a
    24 kHz reference to codes) on a 6 s reference; replicas only.  The
    encode is host-driven like the reference's (resampling on the host, then
    the device stages, codes back): value is the wall-clock rate of
    ov_codec_encode with host samples and host codes (so e2e is the same
    call), max over ranks."""
    import torch

    from omnivoice_b200.codec import Encoder, EncoderConfig
    cfg = EncoderConfig()
    enc = Encoder.synthetic(cfg, seed=1)
    n = int(ENCODE_SECONDS * cfg.sample_rate)
    samples = (0.3 * np.random.default_rng(rank).standard_normal(n)).astype(np.float32)
    for _ in range(max(3, args.warmup)):
        codes = enc.encode(samples)
    torch.cuda.synchronize()
    with ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            codes = enc.encode(samples)
        sec = (time.perf_counter() - t0) / args.steps
    assert codes.shape == (cfg.codebooks, n // cfg.frame_samples)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([sec], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t.item())
    flops = encoder_flops(cfg, n)
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    line = {
        "metric": "reference-audio sec encoded per sec (codec encoder, 6 s reference)",
        "value": world * ENCODE_SECONDS / sec, "unit": "audio_s/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic samples, random-init encoder weights",
        "config": {"workload": f"codec encode of {n} samples ({ENCODE_SECONDS:g} s at 24 kHz) -> "
                               f"8 x {n // cfg.frame_samples} codes",
                   "parallelism": f"replicas{world}", "timing": "host wall clock per call"},
        "roofline": {"bound": "fp32 (CUDA cores)", "achieved": flops / sec / 1e12, "peak": fp32_peak,
                     "unit": "TFLOP/s", "frac": flops / sec / 1e12 / fp32_peak, "traffic": None,
                     "note": "whole encode including host resampling and copies; peak nominal "
                             "(148 SMs x 128 fp32 lanes x 2 x 1.965 GHz), no measured fp32 peak"},
        "e2e": {"value": world * ENCODE_SECONDS / sec, "unit": "audio_s/s",
                "h2d_bytes_per_step": int(samples.nbytes + 4 * int(np.ceil(n * 2 / 3 + 320))),
                "d2h_bytes_per_step": int(codes.nbytes)},
        "gpu_launches": args.steps * (len(cfg.conv_kernels) + 5 + 8 * cfg.layers + 1 + 11 +
                                      2 + 7 * len(cfg.downsampling_ratios) + 2),
        "clocks": clocks.summary(),
    }
    if not args.no_cpu_baseline:
        from oracle import codec_encoder as oe
        shape = oe.EncoderShape()
        weights = oe.synthetic_weights(shape, 1)
        sample = samples[:cfg.sample_rate]
        t0 = time.perf_counter()
        oe.encode(weights, shape, sample)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 1.0 / dt, "unit": "audio_s/s", "cores": os.cpu_count(),
                                "kind": "port",
                                "sample": "oracle/codec_encoder.py (numpy float64) encoding 1 s"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_encode_reference(args, rank):
    """--impl reference --workload encode: the CPU restatement of the
    reference encoder (oracle/codec_encoder.py, numpy; the reference's own
    encoder is HIP code) on a bounded sample: `steps` encodes of 1 s of the
    reference audio.  Rank 0 only."""
    if rank != 0:
        return
    from oracle import codec_encoder as oe
    shape = oe.EncoderShape()
    weights = oe.synthetic_weights(shape, 1)
    sample = (0.3 * np.random.default_rng(0).standard_normal(shape.sample_rate)).astype(np.float32)
    for _ in range(min(args.warmup, 1)):
        oe.encode(weights, shape, sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oe.encode(weights, shape, sample)
    per_second = (time.perf_counter() - t0) / args.steps
    value = 1.0 / per_second
    print(json.dumps({
        "impl": "reference", "metric": "reference-audio sec encoded per sec (codec encoder, 6 s reference)",
        "value": value, "unit": "audio_s/s", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_second * ENCODE_SECONDS * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic samples, random-init encoder weights",
        "config": {"workload": "codec encode of a 6 s reference, sampled as 1 s"},
        "cpu_baseline": {"value": value, "unit": "audio_s/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": "1 s encodes"},
        "e2e": {"value": value, "unit": "audio_s/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


LONGTEXT_CHUNKS = 4        # a 60 s text: four 15 s chunks (synthesizer.cpp:166-178 chunking)
LONGTEXT_FRAMES = 375
LONGTEXT_TEXT = 150


def run_longtext(args, rank, world):
    """--workload longtext: one long text as 4 chunks of 375 frames (60 s of
    audio), generated and decoded by omnivoice_b200.synthesis: chunk 0
    first (its codes carry the voice), chunks 1-3 as one packed batch, each
    chunk decoded by the codec.  value: audio seconds per second (device
    work, wall clock on the host with synchronised calls); the reference's
    chunk-by-chunk order (synthesizer.cpp:180-207) on the same generator and
    codec is reported beside it as `sequential`."""
    import torch

    from omnivoice_b200 import ConditionalInput, DecodingConfig, Generator
    from omnivoice_b200.codec import Codec, CodecConfig
    from omnivoice_b200.synthesis import synthesize_chunks, synthesize_chunks_sequential
    gen = Generator.synthetic(weight_seed=0)
    codec = Codec.synthetic(CodecConfig(), seed=1)
    rng = np.random.default_rng(7 + rank)
    texts = [rng.integers(0, VOCAB, LONGTEXT_TEXT).tolist() for _ in range(LONGTEXT_CHUNKS)]

    def build(i, voice):
        if voice is not None:
            return ConditionalInput.build(texts[voice.index] + texts[i], voice.codes,
                                          LONGTEXT_FRAMES)
        return ConditionalInput.build(texts[i], None, LONGTEXT_FRAMES)

    dec = DecodingConfig()
    seconds = LONGTEXT_CHUNKS * LONGTEXT_FRAMES / FRAME_RATE

    def timed(fn):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / args.steps

    batched = timed(lambda: synthesize_chunks(gen, codec, LONGTEXT_CHUNKS, build, dec, seed=3))
    sequential = timed(lambda: synthesize_chunks_sequential(gen, codec, LONGTEXT_CHUNKS, build,
                                                            dec, seed=3))
    if rank == 0:
        print(json.dumps({
            "metric": "audio-sec synthesised per sec (60 s text, 4 chunks, generate + decode)",
            "value": world * seconds / batched, "unit": "audio_s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": batched * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16/f32",
            "data": "synthetic text ids, random-init generator and codec weights",
            "config": {"workload": f"{LONGTEXT_CHUNKS} chunks x ({LONGTEXT_TEXT} text + "
                                   f"{LONGTEXT_FRAMES} frames), voice carried from chunk 0",
                       "parallelism": f"replicas{world}"},
            "sequential": {"value": world * seconds / sequential, "unit": "audio_s/s",
                           "ms_per_step": sequential * 1e3,
                           "note": "the reference's chunk-by-chunk order on the same kernels"},
            "timing": "host wall clock around synchronised calls (includes host-device copies)"}),
              flush=True)
    gen.close()
    codec.close()


def run_codec_reference(args, rank):
    """--impl reference --workload codec: the CPU restatement of the
    reference decoder (oracle/codec.py, numpy; the reference's own decoder is
    HIP code) on a bounded sample of the chunk: `steps` decodes of 3 frames,
    scaled per frame.  Rank 0 only."""
    if rank != 0:
        return
    from oracle import codec as oc
    shape = oc.CodecShape()
    weights = oc.synthetic_weights(shape, 1)
    sample = np.random.default_rng(0).integers(0, 1024, (8, 3))
    for _ in range(min(args.warmup, 1)):
        oc.decode(weights, shape, sample)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oc.decode(weights, shape, sample)
    per_frame = (time.perf_counter() - t0) / args.steps / 3
    value = 1 / FRAME_RATE / per_frame
    print(json.dumps({
        "impl": "reference", "metric": "audio-sec decoded per sec (codec decoder, 10 s chunk)",
        "value": value, "unit": "audio_s/s", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_frame * CODEC_FRAMES * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic codes, random-init decoder weights",
        "config": {"workload": f"codec decode of {CODEC_FRAMES} frames, sampled as 3 frames"},
        "cpu_baseline": {"value": value, "unit": "audio_s/s", "cores": os.cpu_count(),
                         "kind": "port", "sample": "3-frame decodes, per-frame time scaled"},
        "e2e": {"value": value, "unit": "audio_s/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c5", "codec", "encode",
                                               "longtext"],
                        default="c2")
    parser.add_argument("--noise", choices=["device", "reference"], default="device")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local_rank}"))
        dist = tdist
    try:
        if args.workload == "longtext":
            if args.impl == "reference":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable": "the chunked-synthesis "
                                      "workload has no CPU arm (its sequential order is timed on "
                                      "the GPU as `sequential`)"}), flush=True)
            else:
                run_longtext(args, rank, world)
        elif args.workload == "codec":
            if args.impl == "reference":
                run_codec_reference(args, rank)
            else:
                run_codec(args, rank, world)
        elif args.workload == "encode":
            if args.impl == "reference":
                run_encode_reference(args, rank)
            else:
                run_encode(args, rank, world)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
