"""Benchmark of the B200 motion decoder (mdec frames/s @512x512 f16).

One step = one decode of a 50-frame chunk (f16 weights,
per-frame styles from a seeded random walk, one shared source latent and
feature pyramid, output [50, 3, 512, 512] f32) on every GPU. Multi-GPU runs
(torchrun, one process per GPU) shard frames: each rank decodes its own
50-frame chunk per step (weak scaling). The decoder is a tpmd_group (C++
behind the C ABI): each rank joins the group's NCCL clique, the prepared
weights and the feature pyramid are broadcast once from rank 0 by the group,
and the max over ranks is the group's NCCL all-reduce. No per-step
collective.

value   frames/s over all ranks, device-timed with CUDA events on the launch
        stream, inputs and outputs resident in HBM, max over ranks.
e2e     the same through the host C ABI (tpmd_decode): styles H2D from pinned
        memory and every frame D2H into pinned memory inside the timed region.
roofline  the dominant kernel (largest share of device time, timed live with
        CUDA events around each launch) against MEASURED_PEAKS.json.
cpu_baseline  the CPU oracle (restatement of the reference's CPU decoder) on
        this host's cores, bounded sample, rank 0 at N=1 only.

--impl reference  times that CPU restatement as the reference arm (the
reference itself cannot be built: its ggml submodule is absent).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "talking-portrait.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "mdec frames/s @512x512 f16"
UNIT = "frames/s"
PUBLISHED_FPS = 213.2  # GGML-CUDA f16 mdec, RTX 5070 Ti (reference docs/vulkan-perf.md:143)
ST_IC = (512, 512, 512, 512, 256, 128, 64)
ST_OC = (512, 512, 512, 256, 128, 64, 32)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def kernel_work(name: str, nb: int, esz: int):
    """algorithmic (flops, bytes) of one launch decoding nb frames"""
    if name == "conv1":
        flops = 2.0 * 16 * 512 * 4608 * nb
        byts = nb * 16 * 512 * esz * 2 + 512 * 4608 * esz
        return flops, byts
    if name.startswith("conv2tail_r"):  # conv2 with the level tail fused
        r = int(name[len("conv2tail_r"):])
        f, b = kernel_work(f"conv2_r{r}", nb, esz)
        f2, b2 = kernel_work(f"tail_r{r}", nb, esz)
        j = (r // 8).bit_length() - 1
        # the conv2 output never reaches HBM: drop its write and the tail's read
        return f, b + b2 - 2 * nb * r * r * ST_OC[j] * esz
    for pre, up in (("upconv_r", True), ("conv2_r", False)):
        if name.startswith(pre):
            r = int(name[len(pre):])
            j = (r // 8).bit_length() - 1
            ic, oc = (ST_IC[j], ST_OC[j]) if up else (ST_OC[j], ST_OC[j])
            npix = (r // 2) ** 2 if up else r * r
            n = 4 * oc if up else oc
            flops = 2.0 * npix * n * 9 * ic * nb
            byts = nb * (npix * ic + r * r * oc) * esz + n * 9 * ic * esz
            return flops, byts
    if name.startswith("tail_r"):
        r = int(name[len("tail_r"):])
        j = (r // 8).bit_length() - 1
        oc = ST_OC[j]
        last = j == 6
        per = r * r * oc * esz * (1 if last else 2) + 3 * 4 * r * r * (1 if last else 2)
        per += 2 * 3 * 4 * (r // 2) ** 2 if j else 0
        return 0.0, nb * per + r * r * oc * esz
    return 0.0, 0.0


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU, read
    through NVML (read-only queries) while the timed work runs: `poll_until`
    samples every few ms until the given CUDA event completes, so even a
    short timed region gets samples taken under load. Falls back to an
    nvidia-smi process sampling every 100 ms when NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.nv = None
        self.h = None
        self.proc = None
        self.lines: list[str] = []
        self.rows: list[tuple[float, float, list[str]]] = []

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = None
            try:  # the CUDA device's PCI address names the NVML device exactly
                import torch
                pr = torch.cuda.get_device_properties(self.gpu)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.nv, self.h = nv, h
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            self.nv = None
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                     "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.t = threading.Thread(target=self._read, daemon=True)
                self.t.start()
            except OSError:
                self.proc = None
        return self

    def sample(self):
        if self.nv is None:
            return
        try:
            mhz = float(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            bits = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            return
        self.rows.append((mhz, self.max_mhz, [n for n, b in self.REASONS if bits & b]))

    def poll_until(self, event, period_s: float = 0.003):
        """Sample until `event` (recorded after the timed work) completes."""
        self.sample()
        while not event.query():
            time.sleep(period_s)
            self.sample()

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
        rows = list(self.rows)
        names = [n for n, _ in self.REASONS]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]),
                             [names[i] for i, f in enumerate(parts[4:8]) if f.lower() == "active"]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({r for _, _, rs in rows for r in rs})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows),
                "source": "nvml" if self.rows else "nvidia-smi"}


def cpu_baseline(tensors, feats, styles, budget_s: float = 12.0):
    """oracle sub-pixel graph (the reference CPU path's fast-graph math) on
    all host cores: one warm-up frame, then frames until ~budget_s"""
    import oracle as O
    O.set_threads(os.cpu_count() or 1)  # torchrun exports OMP_NUM_THREADS=1
    dec = O.Decoder(tensors, feats)
    dec.decode(styles[0], mode=1)
    n, t0 = 0, time.perf_counter()
    while n < len(styles) and (time.perf_counter() - t0) < budget_s:
        dec.decode(styles[n % len(styles)], mode=1)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": UNIT, "cores": O.threads(), "kind": "port",
            "sample": f"{n} frames of config 2 (fp32, batch 1, 512x512) after 1 warm-up frame, "
                      f"{dt:.1f} s wall clock, oracle sub-pixel graph"}


def load_synth():
    """the seeded input generators (tpmd/synth.py, numpy only), loaded as a
    plain module so the reference arm imports nothing of the product"""
    import importlib.util
    path = os.path.join(ROOT, "talking-portrait.cpp_b200", "tpmd", "synth.py")
    spec = importlib.util.spec_from_file_location("tp_synth", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def setup_inputs(rank: int, frames: int, scale_for):
    synth = load_synth()
    raw = synth.make_weights(seed=0)
    tensors = synth.fold(raw, scale_for)
    feats = synth.make_feats(seed=0)
    styles = synth.styles_walk(seed=0, n=frames, clip=rank)
    return tensors, feats, styles


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import oracle as O
    tensors, feats, styles = setup_inputs(0, max(8, args.warmup + args.steps), O.scale_for)
    O.set_threads(os.cpu_count() or 1)  # all host threads (torchrun exports OMP_NUM_THREADS=1)
    dec = O.Decoder(tensors, feats)
    for i in range(args.warmup):
        dec.decode(styles[i], mode=1)
    t0 = time.perf_counter()
    for i in range(args.steps):
        dec.decode(styles[(args.warmup + i) % len(styles)], mode=1)
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "config 2 styles, one frame per step (CPU, fp32)",
                       "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": O.threads(), "kind": "port",
                             "sample": f"{args.steps} frames, batch 1, oracle sub-pixel graph; "
                                       "reference unbuildable (ggml submodule absent)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_encoder(args):
    """The motion encoder, one portrait per step on cuda:0, wall clock
    around the blocking tpme_run. `value`: the image H2D, the encoder and the
    small outputs D2H, with the pyramid left on the device (the pipeline's
    path: the decoder takes it through tpmd_set_feats_device); `e2e`: the
    same plus the D2H of all seven feature maps into host arrays. The CPU
    baseline is the oracle's restatement on the host cores."""
    import torch
    import tpmd
    import oracle as O
    from tpmd import synth
    raw = synth.make_encoder_weights(0)
    w = synth.fold(raw, tpmd.scale_for)
    img = synth.make_image(0)
    enc = tpmd.MotionEncoder(0)
    enc.set_tensors(w)
    enc.prepare()
    for _ in range(args.warmup):
        enc.run(img)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        dt = 0.0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            enc.run(img)
            dt += time.perf_counter() - t0
            clk.sample()  # outside the timed call: an NVML query takes host time
        dt /= args.steps
    ms_e2e = dt * 1e3
    t0 = time.perf_counter()
    for _ in range(args.steps):
        enc.run(img, want_feats=False)
    ms_dev = (time.perf_counter() - t0) / args.steps * 1e3
    cpu = None
    if not args.no_cpu_baseline:
        O.set_threads(os.cpu_count() or 1)
        oe = O.Encoder(synth.fold(raw, O.scale_for))
        t0 = time.perf_counter()
        oe.run(img)
        cpu = (time.perf_counter() - t0) * 1e3
    flop = 0.0  # 2*MACs of the convs and linears per portrait
    H = 512
    flop += 2.0 * H * H * 32 * 3
    for i in range(7):
        c, co, h = synth.ENC_IN[i], synth.ENC_OUT[i], H // 2
        flop += 2.0 * H * H * c * c * 9 + 2.0 * h * h * co * c * 9 + 2.0 * h * h * co * c
        H = h
    flop += 2.0 * 512 * 512 * 16 + 2.0 * (4 * 512 * 512 + 20 * 512)
    line = {"metric": "menc ms/portrait @512x512 f32", "value": ms_dev, "unit": "ms",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": "f32", "data": "synthetic (random-init encoder, smooth synthetic image)",
            "config": {"workload": "motion encoder, one 512x512 portrait per step", "global_batch": 1},
            "achieved_tflops": flop / (ms_dev * 1e-3) / 1e12,
            "e2e": {"value": ms_e2e, "unit": "ms", "h2d_bytes_per_step": 3 * 512 * 512 * 4,
                    "d2h_bytes_per_step": 4 * (512 + 20 + 512 + sum(((8 << j) ** 2) * s for j, s in
                                                                   enumerate(synth.ST_OC)))},
            "reference_published_ms": 14.3,
            "clocks": clk.summary(),
            "cpu_baseline": None if cpu is None else {"value": cpu, "unit": "ms", "cores": O.threads(),
                                                      "kind": "port", "sample": "1 portrait"}}
    print(json.dumps(line), flush=True)


def run_fmt(args):
    """The flow-matching sampler of config 4 (8 DiT blocks, d = 1024, 16
    heads, 9 Euler steps with 3-way CFG) on cuda:0: one 50-frame chunk per
    step through tpfm_sample_chunk (host inputs in, motion out), wall clock
    around the blocking call. The CPU baseline is the oracle's restatement
    (one chunk) on the host cores."""
    import tpmd
    import oracle as O
    from tpmd import synth
    cfg = synth.FMT_CONFIG
    w = synth.make_fmt_weights(cfg, 0)
    io = synth.make_fmt_chunk(cfg, 0)
    a = (io["wr"], io["prev_wa"], io["cond_audio"], io["prev_x"], io["x0"], io["emotion"])
    dtype = tpmd.DTYPE_F16 if args.dtype == "f16" else tpmd.DTYPE_F32
    s = tpmd.FmtSampler(cfg, 0, dtype)
    s.set_tensors(w)
    s.prepare()
    for _ in range(args.warmup):
        s.sample(*a)
    with ClockSampler(0) as clk:
        tot = 0.0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            s.sample(*a)
            tot += time.perf_counter() - t0
            clk.sample()  # outside the timed call: an NVML query takes host time
        ms = tot / args.steps * 1e3
    H, T, FF, D = cfg["dim_h"], 60, 4 * cfg["dim_h"], cfg["dim_w"]
    M = 3 * T
    per_block = 2.0 * M * H * (6 * H + 3 * H + H + 2 * FF)
    flop = (cfg["nfe"] - 1) * (cfg["depth"] * per_block + 2.0 * M * H * (2 * H + D) + 2.0 * T * D * H) + \
        2.0 * M * (D + cfg["dim_a"] + cfg["dim_e"]) * H
    cpu = None
    if not args.no_cpu_baseline:
        O.set_threads(os.cpu_count() or 1)
        f = O.Fmt(cfg, w)
        t0 = time.perf_counter()
        f.sample(*a)
        cpu = (time.perf_counter() - t0) * 1e3
    line = {"metric": "fmt ms/chunk (50 frames, 9 steps, 3-way CFG)", "value": ms, "unit": "ms",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": args.dtype, "data": "synthetic (random-init DiT, random chunk inputs)",
            "config": {"workload": "config 4 FMT: 8 blocks, d=1024, 16 heads, 60-frame window",
                       "global_batch": 1},
            "achieved_tflops": flop / (ms * 1e-3) / 1e12,
            "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 4 * D * (1 + 10 + 50 + 10 + 50),
                    "d2h_bytes_per_step": 4 * 50 * D},
            "reference_published_ms": 23.7,
            "clocks": clk.summary(),
            "cpu_baseline": None if cpu is None else {"value": cpu, "unit": "ms", "cores": O.threads(),
                                                      "kind": "port", "sample": "1 chunk"}}
    print(json.dumps(line), flush=True)


def run_audio(args):
    """The audio encoder of config 4 (wav2vec2-base shape: 7 conv layers, 12
    post-norm transformer layers, d = 768) on a 30 s clip to 750 frames on
    cuda:0, through tpae_encode (host audio in, features out), wall clock
    around the blocking call. The CPU baseline is the oracle's restatement
    (one clip) on the host cores."""
    import tpmd
    import oracle as O
    from tpmd import synth
    cfg = synth.AUDIO_CONFIG
    w = synth.make_audio_weights(cfg, 0)
    au = synth.make_audio(30.0, 0)
    S = 750
    e = tpmd.AudioEncoder(cfg, 0)
    e.set_tensors(w)
    e.prepare()
    for _ in range(args.warmup):
        e.encode(au, S)
    with ClockSampler(0) as clk:
        tot = 0.0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            e.encode(au, S)
            tot += time.perf_counter() - t0
            clk.sample()  # outside the timed call: an NVML query takes host time
        ms = tot / args.steps * 1e3
    # GEMM flops: conv stack, feature projection, positional conv, layers, projection
    T, ic, flop = au.size, 1, 0.0
    for i in range(7):
        T = (T - cfg["conv_kernel"][i]) // cfg["conv_stride"][i] + 1
        flop += 2.0 * T * cfg["conv_dim"][i] * ic * cfg["conv_kernel"][i]
        ic = cfg["conv_dim"][i]
    H, F, L = cfg["hidden"], cfg["ffn"], cfg["n_layers"]
    cg = H // cfg["pos_groups"]
    flop += 2.0 * S * ic * H + 2.0 * S * H * cg * cfg["pos_kernel"]
    flop += L * (2.0 * S * H * (4 * H + 2 * F) + 4.0 * S * S * H) + 2.0 * S * L * H * cfg["dim_w"]
    cpu = None
    if not args.no_cpu_baseline:
        O.set_threads(os.cpu_count() or 1)
        o = O.Aud(cfg, w)
        t0 = time.perf_counter()
        o.encode(au, S)
        cpu = (time.perf_counter() - t0) * 1e3
    line = {"metric": "audio encoder ms per 30 s clip (750 frames)", "value": ms, "unit": "ms",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": "f32", "data": "synthetic (random-init wav2vec2-base shape, band-limited speech-like audio)",
            "config": {"workload": "config 4 audio: 30 s of 16 kHz audio -> 750 x 512 features", "global_batch": 1},
            "achieved_tflops": flop / (ms * 1e-3) / 1e12,
            "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 4 * au.size, "d2h_bytes_per_step": 4 * S * 512},
            "clocks": clk.summary(),
            "cpu_baseline": None if cpu is None else {"value": cpu, "unit": "ms", "cores": O.threads(),
                                                      "kind": "port", "sample": "1 clip"}}
    e.close()
    print(json.dumps(line), flush=True)


def run_e2e(args):
    """Config 4: the end-to-end generator on a 30 s clip, real-time factor.
    Rank 0 runs the motion encoder, the audio encoder and the 15 sampler
    chunks (serial by construction: each chunk conditions the next); each
    chunk's styles are broadcast over NCCL as soon as they exist and the
    other ranks decode their share while the next chunk is sampled
    (tpmd.multi.generate_pipelined). On one GPU the public tppl_generate
    decodes each chunk on a worker thread while the next is sampled. Frames
    land in pinned host memory. One step = one clip; the
    time is the max over ranks of the wall clock between barriers;
    RTF = time / 30 s."""
    import torch
    import torch.distributed as dist
    import tpmd
    from tpmd import multi, synth
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    ftype = args.dtype
    dt = tpmd.DTYPE_F16 if ftype == "f16" else tpmd.DTYPE_F32
    raw = synth.make_weights(0)
    w_dec = synth.fold(raw, tpmd.scale_for)
    seconds = 30.0
    audio = synth.make_audio(seconds, 0)
    img = synth.make_image(0)
    n = (audio.size * 25 + 15999) // 16000  # tp_n_frames
    if rank == 0:
        pipe = tpmd.Pipeline(local, ftype, synth.FMT_CONFIG, synth.AUDIO_CONFIG, max_batch=50)
        pipe.set_weights(synth.fold(synth.make_encoder_weights(0), tpmd.scale_for),
                         synth.make_audio_weights(synth.AUDIO_CONFIG, 0),
                         synth.make_fmt_weights(synth.FMT_CONFIG, 0), w_dec)
        dec = pipe.decoder()
    else:
        pipe = None
        dec = tpmd.MotionDecoder(local, dt, 50)
    if world > 1:  # prepared weights once
        t = multi.arena_tensor(dec, 0, dev)
        multi.broadcast_bytes(t, 0)
        torch.cuda.synchronize()
        if rank != 0:
            dec.adopt_arena(0)
    plan = multi.pipeline_plan(n, world)
    frames = torch.empty((max(multi.frames_per_rank(plan, rank), 1), 3, 512, 512), pin_memory=True)
    frames_np = frames.numpy()

    def step():
        if world == 1:  # tppl_generate: each chunk decoded on a worker thread while the next is sampled
            pipe.generate(img, audio, 3, seed=0, out=frames_np)
        else:
            multi.generate_pipelined(rank, world, dev, n, dec, frames, pipe=pipe, image=img, audio=audio,
                                     emotion=3, seed=0)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        dt_s = time.perf_counter() - t0
        if world > 1:
            dt_s = multi.max_over_ranks(dt_s, dev)
        times.append(dt_s)
    sec = float(np.median(times))
    if rank == 0:
        line = {"metric": "end-to-end RTF, 30 s clip (lower is better)", "value": sec / seconds, "unit": "RTF",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
                "scaling": "strong", "dtype": ftype, "data": "synthetic (random-init models, seeded image and "
                "band-limited speech-like audio)",
                "config": {"workload": "config 4: 512x512 portrait + 30 s 16 kHz audio -> 750 frames",
                           "global_batch": n,
                           "parallelism": ("one GPU; each chunk decoded on a second host thread while the next "
                                           "is sampled" if world == 1 else
                                           f"stages 1-3 on rank 0, decode of each chunk overlapped on "
                                           f"{world - 1 if world > 2 else 2} ranks")},
                "x_realtime": seconds / sec,
                "seconds_per_clip": sec, "frames_per_s": n / sec,
                "e2e": {"value": sec / seconds, "unit": "RTF", "h2d_bytes_per_step": 4 * (audio.size + img.size),
                        "d2h_bytes_per_step": n * 3 * 512 * 512 * 4},
                "reference_estimate": "about 0.13 RTF from the published CUDA stage times (15 x 23.7 ms "
                                      "sampler + 750 x 4.69 ms decoder)"}
        print(json.dumps(line), flush=True)
    if pipe is not None:
        dec.close()
        pipe.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_schedule(args):
    """The host decode's schedule on cuda:0 (tpmd_decode / tpmd_decode_rgb24
    with pinned host buffers), config 2's decoder and inputs.

    Prints one JSON line: the device time of one decode of nb frames
    (tpmd_decode_device, CUDA events, median of 5 after 2 warm-ups) for
    several nb, which gives the fixed and per-frame parts of a decode; the
    device-to-host copy time of nb f32 frames into pinned memory; and the
    host-buffer throughput of a 50-frame call (10 calls after 1 warm-up) with
    the split schedule and with TPMD_NO_SPLIT (whole-decode sub-batches), for
    f32 and RGB24 frames, alternating so both see the same box state."""
    import torch
    import tpmd
    tensors, feats, styles = setup_inputs(0, args.batch, tpmd.scale_for)
    nb_max = args.batch
    dec = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, max_batch=nb_max)
    dec.set_tensors(tensors)
    dec.prepare()
    dec.set_feats(feats)
    st = torch.cuda.Stream()
    s_d = torch.from_numpy(np.ascontiguousarray(styles)).cuda()
    f_d = torch.empty((nb_max, 3, 512, 512), device="cuda")
    out = {"path": "schedule", "config": f"config 2 decoder, {nb_max}-frame calls, f16", "decode_ms": {},
           "d2h_ms": {}, "host_fps": {}}
    for nb in sorted({1, 2, 4, 8, 16, 25, 32, nb_max}):
        if nb > nb_max:
            continue
        ts = []
        for _ in range(7):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            dec.decode_device(s_d.data_ptr(), nb, f_d.data_ptr(), st.cuda_stream)
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        out["decode_ms"][nb] = float(np.median(ts[2:]))
    f_h = torch.empty((nb_max, 3, 512, 512), pin_memory=True)
    r_h = torch.empty((nb_max, 512, 512, 3), dtype=torch.uint8, pin_memory=True)
    for nb in sorted({1, 10, nb_max}):
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            with torch.cuda.stream(st):
                f_h[:nb].copy_(f_d[:nb], non_blocking=True)
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        out["d2h_ms"][nb] = float(np.median(ts[1:]))
    s_h = torch.from_numpy(np.ascontiguousarray(styles)).pin_memory()
    for rep in range(2):
        for fmt in ("f32", "rgb24"):
            for plan in ("split", "no_split"):
                if plan == "no_split":
                    os.environ["TPMD_NO_SPLIT"] = "1"
                call = (lambda: dec.decode_ptr(s_h.data_ptr(), nb_max, f_h.data_ptr())) if fmt == "f32" else \
                       (lambda: dec.decode_rgb24_ptr(s_h.data_ptr(), nb_max, r_h.data_ptr()))
                call()
                t0 = time.perf_counter()
                for _ in range(10):
                    call()
                out["host_fps"].setdefault(f"{fmt}_{plan}", []).append(10 * nb_max / (time.perf_counter() - t0))
                os.environ.pop("TPMD_NO_SPLIT", None)
    print(json.dumps(out), flush=True)


def run_ops(args):
    """BASELINE config 1, the decoder's op-level sweep on cuda:0.

    (b) tpk_bilinear_gather over C in {32..512} x H=W in {8..512}, grid
        uniform in [-1.1, 1.1], f32 and f16 feats; (c) tpk_im2col_cf 3x3 pad 1
        on the same shapes (f16 and f32 destinations). Each launch is timed
        alone with CUDA events on its stream after a 256 MB L2 flush; GB/s are
        compulsory bytes (gather: C*H*W*sizeof(feat) + 8N + 4CN with N = H*W;
        im2col: 4*IC*IW*IH + 9*IC*OW*OH*sizeof(dst)) over the median launch
        time, as a fraction of MEASURED_PEAKS.json's copy bandwidth.
    (a) the modulated convs of every level at batch 1..64: a decode of that
        many frames with live per-kernel CUDA-event timing
        (tpmd_profile_begin/end); TFLOP/s per up-conv / conv2 launch against
        the measured bf16 peak."""
    import torch
    import tpmd
    from tpmd import synth
    hbm, tf_burst, tf_sus, src = peaks()
    dev = torch.device("cuda", 0)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(0)

    def timed(fn, reps=5):
        ts = []
        for i in range(reps + 1):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            if i:
                ts.append(e0.elapsed_time(e1) / 1e3)
        return float(np.median(ts))

    chans = (32, 64, 128, 256, 512)
    sizes = (8, 16, 32, 64, 128, 256, 512)
    if args.shape:  # one shape only (e.g. for a profiler capture), no modconv sweep
        c1, h1 = (int(v) for v in args.shape.split(","))
        chans, sizes = (c1,), (h1,)
    gather, im2col = [], []
    for C in chans:
        for H in sizes:
            N = H * H
            grid = torch.from_numpy(rng.uniform(-1.1, 1.1, (N, 2)).astype(np.float32)).to(dev)
            out = torch.empty((N, C), dtype=torch.float32, device=dev)
            for dt, es in ((torch.float32, 4), (torch.float16, 2)):
                feat = torch.randn((N, C), device=dev).to(dt)
                t = timed(lambda: tpmd.bilinear_gather(feat, H, H, grid, out, stream=stream.cuda_stream))
                b = C * N * es + 8 * N + 4 * C * N
                gather.append({"C": C, "H": H, "feat": "f16" if es == 2 else "f32", "us": t * 1e6,
                               "GBps": b / t / 1e9, "frac": b / t / 1e9 / hbm,
                               "tap_GBps": 4 * C * N * es / t / 1e9})
                del feat
            src_t = torch.randn((N, C), device=dev)
            for dt, es in ((torch.float16, 2), (torch.float32, 4)):
                dst = torch.empty((N, 9 * C), dtype=dt, device=dev)
                t = timed(lambda: tpmd.im2col_cf(src_t, C, H, H, 1, dst, stream=stream.cuda_stream))
                b = 4 * C * N + 9 * C * N * es
                im2col.append({"C": C, "H": H, "dst": "f16" if es == 2 else "f32", "us": t * 1e6,
                               "GBps": b / t / 1e9, "frac": b / t / 1e9 / hbm})
                del dst
            del src_t, out, grid
    torch.cuda.synchronize()
    # (a) modconv per level at batch 1..64 through live per-kernel timing
    raw = synth.make_weights(seed=0)
    tensors = synth.fold(raw, tpmd.scale_for)
    feats = synth.make_feats(seed=0)
    modconv = []
    for B in (() if args.shape else (1, 2, 4, 8, 16, 32, 64)):
        d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, B)
        d.set_tensors(tensors)
        d.prepare()
        d.set_feats(feats)
        st = torch.from_numpy(synth.styles_walk(seed=0, n=B)).to(dev)
        fr = torch.empty((B, 3, 512, 512), device=dev)
        for _ in range(2):
            d.decode_device(st.data_ptr(), B, fr.data_ptr(), stream.cuda_stream)
        d.profile_begin()
        for _ in range(3):
            d.decode_device(st.data_ptr(), B, fr.data_ptr(), stream.cuda_stream)
        prof = d.profile_end()
        for name, (n, ms) in prof.items():
            if name.startswith(("upconv_r", "conv2_r", "conv2tail_r")) or name == "conv1":
                flops, _ = kernel_work(name, B, 2)
                modconv.append({"batch": B, "kernel": name, "us": ms / n * 1e3,
                                "TFLOPs": flops / (ms / n / 1e3) / 1e12,
                                "frac": flops / (ms / n / 1e3) / 1e12 / tf_burst})
        d.close()
        del st, fr
    g_f16 = [g for g in gather if g["feat"] == "f16"]
    line = {"metric": "decoder op sweep (config 1)", "unit": "GB/s | TFLOP/s", "n_gpus": 1,
            "data": "synthetic (N(0,1) maps, grid uniform in [-1.1, 1.1]; random-init decoder)",
            "peaks": {"hbm_gbs": hbm, "bf16_tflops_burst": tf_burst, "source": src},
            "gather_best_frac": max(g["frac"] for g in gather),
            "gather_f16_median_frac_large": float(np.median([g["frac"] for g in g_f16 if g["H"] >= 128]))
            if any(g["H"] >= 128 for g in g_f16) else None,
            "im2col_best_frac": max(g["frac"] for g in im2col),
            "gather": gather, "im2col": im2col, "modconv": modconv}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=50)
    ap.add_argument("--dtype", default="f16", choices=["f16", "f32"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shape", default="",
                    help="--path ops: only this 'C,H' shape (gather and im2col), no modconv sweep")
    ap.add_argument("--clip", type=int, default=0,
                    help="config 3: decode a clip of this many frames sharded across ranks per step")
    ap.add_argument("--path", default="decoder",
                    choices=["decoder", "encoder", "fmt", "audio", "e2e", "ops", "schedule"],
                    help="encoder: time the motion encoder (once per portrait); fmt: time the "
                         "flow-matching sampler (one 50-frame chunk per step); audio: the audio encoder "
                         "(one 30 s clip per step); schedule: the host decode's schedule (decode time "
                         "by batch, frame copy time, host-buffer throughput with and without the split "
                         "schedule); one GPU")
    args = ap.parse_args()
    if args.path == "encoder":
        run_encoder(args)
        return
    if args.path == "fmt":
        run_fmt(args)
        return
    if args.path == "audio":
        run_audio(args)
        return
    if args.path == "e2e":
        run_e2e(args)
        return
    if args.path == "ops":
        run_ops(args)
        return
    if args.path == "schedule":
        run_schedule(args)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    import tpmd
    from tpmd import multi, synth

    torch.cuda.set_device(local)
    nccl_id = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        box = [tpmd.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)  # the C++ group's NCCL clique id
        nccl_id = box[0]
    nb = args.batch
    tensors, feats, styles = setup_inputs(rank, nb, tpmd.scale_for)
    dtype = tpmd.DTYPE_F16 if args.dtype == "f16" else tpmd.DTYPE_F32
    # the decoder group (tpmd_group_*, C++ behind the C ABI): this rank's GPU
    # in a clique of `world`; weights and feats are prepared on rank 0 and
    # broadcast once by the group's own NCCL communicator
    group = tpmd.MotionDecoderGroup((local,), dtype, nb, rank=rank, nranks=world, nccl_id=nccl_id)
    if rank == 0:
        group.set_tensors(tensors)
    group.prepare()
    group.set_feats(feats if rank == 0 else None)
    dec = group.member(0)

    stream = torch.cuda.Stream()  # the launch stream; CUDA events are recorded on it
    if args.clip:
        # config 3: a clip of args.clip frames sharded by frame across ranks
        lo, hi = tpmd.shard_range(args.clip, world, rank)
        clip_styles = synth.styles_walk(seed=0, n=args.clip)[lo:hi]
        styles = clip_styles if hi > lo else styles[:1]
        parts = multi.sub_batches(0, len(styles), nb)
    else:
        parts = [(0, nb)]
    s_d = torch.from_numpy(np.ascontiguousarray(styles)).cuda()
    f_d = torch.empty((max(b - a for a, b in parts), 3, 512, 512), device="cuda")
    torch.cuda.synchronize()

    def step():
        for a, b in parts:
            dec.decode_device(s_d.data_ptr() + a * 512 * 4, b - a, f_d.data_ptr(), stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- device-timed region
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        clk.poll_until(e1)
        torch.cuda.synchronize()
    barrier()
    ms = group.max(e0.elapsed_time(e1))  # max over ranks
    frames_per_step = args.clip if args.clip else world * nb
    value = frames_per_step * args.steps / (ms / 1000.0)

    # ---- end to end through the host C ABI (pinned buffers)
    n_mine = len(styles) if args.clip else nb
    s_h = torch.from_numpy(np.ascontiguousarray(styles[:n_mine])).pin_memory()
    f_h = torch.empty((n_mine, 3, 512, 512), pin_memory=True)
    dec.decode_ptr(s_h.data_ptr(), n_mine, f_h.data_ptr())
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dec.decode_ptr(s_h.data_ptr(), n_mine, f_h.data_ptr())
    dt = group.max(time.perf_counter() - t0)
    e2e = frames_per_step * args.steps / dt

    # ---- the same with the reference's output format (RGB24 bytes, converted
    # on the GPU: a quarter of the bytes cross to the host)
    r_h = torch.empty((n_mine, 512, 512, 3), dtype=torch.uint8, pin_memory=True)
    dec.decode_rgb24_ptr(s_h.data_ptr(), n_mine, r_h.data_ptr())
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dec.decode_rgb24_ptr(s_h.data_ptr(), n_mine, r_h.data_ptr())
    dt = group.max(time.perf_counter() - t0)
    e2e_rgb = frames_per_step * args.steps / dt

    # ---- live per-kernel timing (untimed pass) for the roofline
    dec.profile_begin()
    for _ in range(2):
        step()
    prof = dec.profile_end()
    hbm, tf_burst, tf_sus, src = peaks()
    esz = 2 if dtype == tpmd.DTYPE_F16 else 4
    total = sum(v[1] for v in prof.values())
    top = max(prof.items(), key=lambda kv: kv[1][1])
    name, (launches, tot_ms) = top
    avg_s = tot_ms / launches / 1000.0
    flops, byts = kernel_work(name, nb, esz)
    t_tensor = flops / (tf_sus * 1e12)
    t_hbm = byts / (hbm * 1e9)
    if t_tensor >= t_hbm:
        roof = {"bound": "tensor", "achieved": flops / avg_s / 1e12, "peak": tf_sus, "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": byts / avg_s / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["kernel"] = name
    roof["share"] = tot_ms / total
    roof["peak_source"] = src + (" sustained bf16" if roof["bound"] == "tensor" else " copy")
    traffic = None
    tp = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tp):
        # ncu DRAM bytes of this kernel from a batch-8 capture, scaled to this
        # launch: the feats are read once per launch, the rest per frame. Used
        # only while the kernel's sources are the ones captured (their hash)
        tj = json.load(open(tp))
        if tj.get("kernel") == name and tj.get("conv") == ("tc" if dec_uses_tc() else "simt") and \
                tj.get("source_sha256") == conv_source_hash():
            traffic = tj["fixed_bytes"] + tj["bytes_per_frame"] * nb
    roof["traffic"] = traffic
    roof["algorithmic_bytes"] = byts
    kernels = {k: {"launches": v[0], "ms": round(v[1], 4), "share": round(v[1] / total, 4)}
               for k, v in sorted(prof.items(), key=lambda kv: -kv[1][1])}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(tensors, feats, styles)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.clip else "weak", "vs_baseline": value / PUBLISHED_FPS,
            "dtype": args.dtype,
            "data": "synthetic (random-init decoder, smooth N(0,1) feats, random-walk styles)",
            "config": {"workload": (f"config 3: {args.clip}-frame clip sharded by frame, sub-batches of "
                                    f"<= {nb}, f16 weights, 512x512") if args.clip else
                                   "config 2: 50-frame chunk per GPU, f16 weights, 512x512",
                       "global_batch": frames_per_step, "frames_per_gpu_per_step": n_mine,
                       "parallelism": f"frame-sharded x{world}",
                       "l2": "no flush: per-step working set (~2 GB activations) exceeds the 126 MB L2",
                       "conv": "tcgen05" if dec_uses_tc() else "simt"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": frames_per_step * 512 * 4,
                    "d2h_bytes_per_step": frames_per_step * 3 * 512 * 512 * 4},
            "e2e_rgb24": {"value": e2e_rgb, "unit": UNIT, "h2d_bytes_per_step": frames_per_step * 512 * 4,
                          "d2h_bytes_per_step": frames_per_step * 3 * 512 * 512,
                          "api": "tpmd_decode_rgb24 (frames as the reference CLI's RGB24 bytes)"},
            "gpu_launches": sum(dec.kernel_launches(b - a) for a, b in parts) * args.steps * world,
            "roofline": roof, "kernels": kernels, "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    barrier()
    group.close()
    if world > 1:
        dist.destroy_process_group()


def conv_source_hash() -> str:
    """sha256 over the tcgen05 conv kernel's sources (kernels_conv_tc.cu,
    tc_ptx.cuh): the key of the recorded ncu traffic figure"""
    import hashlib
    h = hashlib.sha256()
    for f in ("kernels_conv_tc.cu", "tc_ptx.cuh"):
        with open(os.path.join(ROOT, "talking-portrait.cpp_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def dec_uses_tc() -> bool:
    return os.environ.get("TPMD_CONV", "tc" if TC_DEFAULT else "simt") == "tc"


TC_DEFAULT = True

if __name__ == "__main__":
    main()
