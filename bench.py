"""×realtime of the Mel-Band RoFormer separation path on 1..8 B200s (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json configs[0] model, native context): Mel-Band RoFormer dim 384, depth 6,
8×64 heads, 60 mel bands, n_fft 2048, hop 441, chunk 352800, overlap 4, one stem, seeded
N(0, 0.02) weights; each GPU separates its own synthetic stereo track (Gaussian σ = 0.1,
44.1 kHz, ``--seconds`` long, seed = 1000 + rank). A step is the whole pipeline over that
track: chunk gather → STFT → model → complex mask + iSTFT → overlap-add → crop. Chunks are
independent, so ranks shard the work with no collective ("scaling": "weak").

* ``value``: audio seconds separated per wall second over all ranks, with the PCM already in
  HBM (``ancha_separate_device``), timed with CUDA events on the launch stream, max over
  ranks. The working set (≈0.5 GB of weights, ≈0.7 GB of activations per chunk) exceeds the
  126 MB L2, so no extra flush runs between steps.
* ``e2e``: the same through ``ancha_separate_pcm`` (host PCM in, host stems out, host↔device
  copies inside the timed region).
* ``roofline``: the dominant kernel re-launched alone with CUDA events.
* ``attention``: BASELINE config 2, the fused attention alone (time axis T = 801 / 1601 / 3201
  and the band axis S = 60) in the bench dtype, and the fp32 (FFMA) variant at T = 801.
* ``strong_track``: the same Mel-Band RoFormer on ONE 180 s track (96 chunks) split over the
  ranks (``ancha_b200.distributed``: each rank separates its chunk range from the PCM slice it
  needs, sends only the chunk-overlap halo of its span to the rank that owns those samples,
  divides its owned range on its GPU, then one gather of the stems to rank 0), host PCM in and
  host stems out on rank 0, CUDA events per rank around the whole call, max over ranks,
  ``"scaling": "strong"``. At N=1 it runs ``ancha_separate_pcm``.
* ``fp32``: the ``value`` pipeline and track in fp32, the reference's arithmetic and BASELINE
  config 1's dtype (transformer GEMMs on the tensor cores through three-plane bf16 splits, the
  rest on FFMA kernels), PCM in HBM, CUDA events, max over ranks.
* ``config3``: BASELINE config 3, BS-RoFormer dim 512, depth 12, 8×64 heads, 62 bands, hop 512,
  in f16 (the config names bf16, which misses the 50 dB tolerance on this network), one 180 s track (chunk 352800, overlap 2 → 47 chunks) split over the ranks the same way,
  ``"scaling": "strong"``.
* ``config4``: BASELINE config 4, the MDX23C inst_voc_hq2 forward in bf16, 16 chunks per GPU
  (4 calls of batch 4) on spectra in HBM: ms, TFLOP/s against the measured bf16 peak, and
  model-only ×realtime (0.74 s of new audio per chunk at overlap 8).
* ``config5`` (``--no-config5`` skips it): BASELINE config 5, a synthetic classic MDX-Net
  (TFC-TDF v1) ONNX graph (``ancha_b200.mdx_net``; n_fft 6144, hop 1024, dim_f 3072, dim_t 256)
  through the classic MDX executor with conv_gemm, bf16 and fp32: model-only ms and TFLOP/s for
  16 tiles per GPU (4 calls of batch 4), and end to end four-minute tracks through
  ``ancha_mdx_separate_pcm`` (bf16): each rank's share of 64 tracks, at most 8 of them timed,
  aggregate ×realtime from the slowest rank's summed separation time.
* ``cpu_baseline``: the numpy oracle (f32, all host cores) on one native chunk, median of 3
  after one warm-up (rank 0, N=1). It is a port of the reference CPU path, not the reference's
  own Burn CPU backend, so ratios against it are ratios against the numpy port.
* ``--impl reference`` times that CPU port the same way (the reference itself is Rust and
  cannot be built offline).
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
sys.path.insert(0, ROOT)

METRIC = "×realtime (audio s/wall s) Mel-RoFormer at 1/2/4/8 B200; fused-attn TFLOP/s vs peak"
SR, CHUNK, OVERLAP, HOP = 44100, 352800, 4, 441


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--precision", default="f16", choices=["f16", "bf16", "f32"])
    p.add_argument("--seconds", type=float, default=30.0)
    p.add_argument("--batch", type=int, default=0, help="chunks per model call (0 = the library's balanced default)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--package", default=os.environ.get("ANCHA_BENCH_PACKAGE", "/tmp/ancha_bench/mel-seed0"))
    p.add_argument("--no-config3", action="store_true")
    p.add_argument("--no-config4", action="store_true")
    p.add_argument("--no-config5", action="store_true")
    p.add_argument("--pipeline-only", action="store_true",
                   help="run only the warm-up and timed pipeline steps (for launch-list captures)")
    return p.parse_args()


def config5(local: int, world: int, rank: int, dist, steps: int = 2):
    """BASELINE config 5 (see the module docstring); returns the JSON block on rank 0."""
    import torch
    from ancha_b200.mdx import Graph
    from ancha_b200.mdx_net import MdxNetConfig, forward_flops, tfc_tdf_v1
    c = MdxNetConfig()
    onnx = tfc_tdf_v1(c, seed=0)
    g = torch.Generator(device="cuda").manual_seed(6000 + rank)
    x = torch.randn(16, 4, c.dim_f, c.dim_t, device="cuda", generator=g) * 0.1
    out = torch.empty_like(x)

    def max_over_ranks(v):
        if dist:
            t = torch.tensor([v], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t.item())
        return v

    # End to end: this rank's share of the 64 tracks, at most 8 of them timed (one 4-minute
    # track takes about a second on one GPU), so the leg stays near ten seconds at any N.
    ms, e2e_s, tracks = {}, None, min(8, 64 // world)
    for mode in ("bf16", "f32"):
        graph = Graph(onnx, local, True, gemm=mode)

        def step():
            for i in range(0, 16, 4):
                out[i:i + 4] = graph.forward(x[i:i + 4])

        step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        ms[mode] = max_over_ranks(a.elapsed_time(b) / steps)
        assert bool(torch.isfinite(out).all())
        if mode == "bf16":
            # End to end: this rank's share of 64 four-minute tracks, host PCM in and host
            # predicted / residual out (Inst HQ 2's STFT, mdx.rs:36-93), separation time summed.
            opts = dict(n_fft=6144, hop=1024, bins=c.dim_f, frames=c.dim_t, compensate=1.033, batch=4)
            graph.separate_pcm(track(10.0, 7000 + rank), **opts)  # warm-up
            total = 0.0
            for i in range(tracks):
                total += graph.separate_pcm(track(240.0, 7100 + 64 * rank + i), **opts)[2]
            e2e_s = max_over_ranks(total)
        graph.close()
    if rank != 0:
        return None
    flops = forward_flops(c, 16)
    new_audio = 16 * (1024 * (c.dim_t - 1) - 6144) / SR  # UVR default step: chunk − n_fft per tile
    return {"workload": f"classic MDX-Net (TFC-TDF v1, synthetic ONNX, growth {c.growth}, {c.scales} scales) "
                        f"forward, 16 tiles [4, {c.dim_f}, {c.dim_t}] per GPU as 4 calls of batch 4, x{world} GPU(s)",
            "ms_per_16_tiles": ms, "tflop_per_16_tiles": flops / 1e12,
            "tflops_per_gpu": {m: flops / (v / 1e3) / 1e12 for m, v in ms.items()},
            "tflops_frac_bf16": flops / (ms["bf16"] / 1e3) / 1e12 / peaks()[1],
            "x_realtime_model_only": {m: new_audio * world / (v / 1e3) for m, v in ms.items()},
            "e2e": {"tracks_timed": tracks * world, "of_tracks": 64, "seconds_each": 240.0, "slowest_rank_s": e2e_s,
                    "x_realtime": tracks * world * 240.0 / e2e_s, "dtype": "bf16",
                    "timing": "summed separation time per rank (ancha_mdx_separate_pcm, host PCM in, host "
                              "outputs out), max over ranks"},
            "note": "conv_gemm mode: convolutions, 2x2 transposed convolutions and TDF MatMuls as GEMMs"}


def one_track(model, planes, chunk: int, overlap: int, local: int, world: int, dist, steps: int):
    """One track split over the ranks (``ancha_b200.distributed``: each rank separates its chunk
    range from the PCM slice it needs, the chunk-overlap halos go to their owners over NCCL, each
    rank divides its owned range on its GPU, one gather brings the stems to rank 0), or on one GPU
    through ``ancha_separate_pcm``. Host PCM in, host stems out on rank 0. Returns the median over
    ``steps`` of the per-step time (s), each step timed with CUDA events on the rank's stream around
    the whole call, max over ranks, and rank 0's stems."""
    import torch

    from ancha_b200.distributed import ChunkPlan, GpuShard, separate_distributed
    from ancha_b200.model import separate_pcm
    plan = ChunkPlan.of(planes.shape[1], chunk, overlap)
    ops = GpuShard(model) if dist else None
    rank = dist.get_rank() if dist else 0
    stems = pinned((model.stems, 2, planes.shape[1])) if rank == 0 else None

    def run():
        if dist:
            return separate_distributed(planes, plan, ops, model.stems * 2, out=stems)
        return separate_pcm([model], planes, chunk, overlap, out=stems)[0]

    out = run()
    times = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(steps):
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        out = run()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=f"cuda:{local}")
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(float(t.item()))
    return float(np.median(times)), out, plan


def config3(local: int, world: int, rank: int, dist, steps: int = 2):
    """BASELINE config 3 (see the module docstring); returns the JSON block on rank 0."""
    from ancha_b200.config import ModelConfig
    from ancha_b200.model import Roformer
    pkg = "/tmp/ancha_bench/bs512-seed0"
    ensure_package(pkg, rank if world == 1 else int(os.environ.get("LOCAL_RANK", "0")),
                   ModelConfig.bs_roformer_512())
    # f16 operands: BASELINE names bf16, whose 8-bit mantissa caps this seeded network near 40 dB
    # (tests/test_gpu_model.py), below the 50 dB tolerance; f16 runs at the same tensor-core rate.
    model = Roformer(pkg, local, "f16")
    planes = pinned_track(180.0, 3000)
    t, out, plan = one_track(model, planes, model.chunk_samples, model.overlap, local, world, dist, steps)
    model.close()
    if rank != 0:
        return None
    assert out is not None and np.all(np.isfinite(out))
    return {"workload": "bs-roformer dim512 depth12 8x64 heads, 62 bands, hop 512, f16, 180 s track, "
                        f"chunk {plan.chunk_samples}, overlap {plan.overlap} ({plan.chunks} chunks) sharded "
                        f"over {world} GPU(s)", "value": 180.0 / t, "unit": "×realtime",
            "seconds_per_track": t, "steps": steps, "scaling": "strong", "dtype": "f16",
            "timing": "CUDA events per rank around the whole call (host PCM in, host stems out on rank 0), "
                      "max over ranks, median of steps"}


def fp32_leg(package: str, local: int, world: int, rank: int, dist, planes, d_planes, steps: int = 2):
    """The same pipeline and track as ``value`` in fp32 (the reference's arithmetic and BASELINE
    config 1's dtype): PCM in HBM, CUDA events, max over ranks."""
    import ctypes as C

    import torch

    from ancha_b200 import _native as N
    from ancha_b200.model import Roformer
    model = Roformer(package, local, "f32")
    samples = planes.shape[1]
    d_stems = torch.empty((model.stems, 2, samples), dtype=torch.float32, device=f"cuda:{local}")
    stream = torch.cuda.Stream()
    L = N.lib()

    def step():
        N.check(L.ancha_separate_device(model.handle, d_planes.data_ptr(), samples, CHUNK, OVERLAP, 0,
                                        d_stems.data_ptr(), C.c_void_p(stream.cuda_stream)))

    with torch.cuda.stream(stream):
        step()
        N.check(L.ancha_separate_status(model.handle, C.c_void_p(stream.cuda_stream)))
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        N.check(L.ancha_separate_status(model.handle, C.c_void_p(stream.cuda_stream)))
    t = torch.tensor([e0.elapsed_time(e1) / 1e3 / steps], device=f"cuda:{local}")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    model.close()
    if rank != 0:
        return None
    sec = float(t.item())
    return {"workload": "the value workload (mel-band-roformer, native context, one 30 s track per GPU) in fp32",
            "value": world * samples / SR / sec, "unit": "×realtime", "ms_per_step": sec * 1e3, "steps": steps,
            "dtype": "f32", "scaling": "weak",
            "kernels": "transformer and mask-head GEMMs and the attention of both axes on the tensor cores "
                       "with three-plane bf16 operand splits (six plane products, f32 accumulation); band split "
                       "on the FFMA kernel"}


def mel_track(model, local: int, world: int, rank: int, dist, precision: str, steps: int = 3):
    """The Mel-Band RoFormer on ONE 180 s track split over the ranks (strong scaling of the
    headline model at native context: chunk 352800, overlap 4, 96 chunks)."""
    planes = pinned_track(180.0, 4000)
    t, out, plan = one_track(model, planes, CHUNK, OVERLAP, local, world, dist, steps)
    if rank != 0:
        return None
    assert out is not None and np.all(np.isfinite(out))
    return {"workload": f"mel-band-roformer dim384 depth6, {precision}, one 180 s track, chunk {CHUNK}, "
                        f"overlap {OVERLAP} ({plan.chunks} chunks) sharded over {world} GPU(s)",
            "value": 180.0 / t, "unit": "×realtime", "seconds_per_track": t, "steps": steps, "scaling": "strong",
            "dtype": precision, "h2d_bytes_per_step": int(planes.nbytes),
            "d2h_bytes_per_step": int(model.stems * 2 * planes.shape[1] * 4),
            "timing": "CUDA events per rank around the whole call (host PCM in, host stems out on rank 0), "
                      "max over ranks, median of steps"}


def config4(local: int, world: int, rank: int, dist, steps: int = 3):
    """the MDX23C inst_voc_hq2 forward (TFC-TDF v3 U-Net, 128 channels,
    growth 128, 5 scales, 2 blocks per scale, bottleneck factor 4; dim_f 4096 × dim_t 256),
    bf16, seeded synthetic weights, 16 chunks per GPU as 4 calls of batch 4 (the reference's
    batch limit, mdx23c.rs:428-431) on spectra already in HBM; CUDA events, max over ranks."""
    import torch
    from ancha_b200.mdx23c import Mdx23c, forward_flops, inst_voc_hq2, random_tensors, write_package
    c = inst_voc_hq2()
    pkg = "/tmp/ancha_bench/mdx23c-seed0"
    if rank == 0 or int(os.environ.get("LOCAL_RANK", "0")) == 0:
        if not os.path.exists(os.path.join(pkg, "manifest.json")):
            write_package(pkg + ".tmp", c, random_tensors(c, seed=0))
            os.replace(pkg + ".tmp", pkg)
    if dist:
        dist.barrier()
    model = Mdx23c(pkg, local, "bf16")
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    x = torch.randn(16, 4, c["bins"], c["frames"], device="cuda", generator=g) * 0.1
    out = torch.empty(16, 8, c["bins"], c["frames"], device="cuda")

    def step():
        for i in range(0, 16, 4):
            out[i:i + 4] = model.forward(x[i:i + 4])

    step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        step()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    assert bool(torch.isfinite(out).all())
    # End to end through ancha_mdx23c_separate_pcm: a 60 s host track in, host stems out
    # (UVR chunks, STFT 8192 / hop 1024, network, iSTFT, overlap-add on the GPU), wall clock.
    pcm = track(60.0, 5000 + rank)
    model.separate_pcm(pcm[:, :44100 * 8])  # warm-up (workspace for batch 4)
    e2e_s = min(model.separate_pcm(pcm)[1] for _ in range(2))
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    model.close()
    if rank != 0:
        return None
    flops = forward_flops(c, 16, c["frames"])
    new_audio = 16 * c["hop"] * (c["frames"] - 1) / c["overlap"] / c["sample_rate"]
    return {"workload": "mdx23c inst_voc_hq2 forward, bf16, 16 chunks [4, 4096, 256] per GPU as 4 calls "
                        f"of batch 4, x{world} GPU(s)",
            "ms_per_16_chunks": ms, "chunks_per_s": 16 * world / (ms / 1e3),
            "tflops_per_gpu": flops / (ms / 1e3) / 1e12,
            "tflops_frac": flops / (ms / 1e3) / 1e12 / peaks()[1],
            "x_realtime_model_only": new_audio * world / (ms / 1e3),
            "note": "x_realtime_model_only counts the 0.74 s of new audio per chunk at overlap 8; "
                    "STFT / iSTFT / overlap-add not included",
            "e2e": {"value": 60.0 * world / e2e_s, "unit": "×realtime", "seconds_per_60s_track": e2e_s,
                    "timing": "wall clock of ancha_mdx23c_separate_pcm per rank (host PCM in, host stems "
                              "out), best of 2, max over ranks"},
            "scaling": "weak", "dtype": "bf16"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            m = json.load(fh)
        return m["hbm_gbs"], m["bf16_tflops"], m.get("bf16_tflops_sustained", m["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def ensure_package(path: str, rank: int, config=None):
    from ancha_b200 import synthetic
    from ancha_b200.config import ModelConfig
    done = os.path.join(path, "manifest.json")
    if rank == 0 and not os.path.exists(done):
        tmp = path + f".tmp{os.getpid()}"
        synthetic.seeded_package(tmp, config or ModelConfig.mel_karaoke())
        os.makedirs(os.path.dirname(path), exist_ok=True)
        os.replace(tmp, path)
    while not os.path.exists(done):
        time.sleep(0.5)


def track(seconds: float, seed: int):
    n = int(round(seconds * SR))
    return (np.random.default_rng(seed).standard_normal((2, n)) * 0.1).astype(np.float32)


def pinned(shape):
    """A float32 host array in page-locked memory (the host side of the end-to-end legs)."""
    import torch
    return torch.empty(shape, dtype=torch.float32, pin_memory=True).numpy()


def pinned_track(seconds: float, seed: int):
    planes = track(seconds, seed)
    buf = pinned(planes.shape)
    buf[...] = planes
    return buf


def plan_chunks(samples: int, chunk=CHUNK, overlap=OVERLAP):
    step = chunk // overlap
    border = chunk - step
    border = border if samples > 2 * border else 0
    length = samples + 2 * border
    return len(range(0, length, step)), length


def effective_batch(chunks: int, batch: int) -> int:
    """The chunks per model call the library uses (runtime.cpp default_batch for 0)."""
    if batch > 0:
        return batch
    batches = max(1, -(-chunks // 8))
    return max(1, -(-chunks // batches))


def launches_per_step(chunks: int, batch: int, depth=6, stems=1, mask_layers=2, mel=True, fused=True):
    """Kernels of this library launched per step, from the pipeline structure (checked against
    the ncu launch list in profiles/bench_launches_mel_native.md: 74 per 4-chunk batch + 1)."""
    if fused:  # 16-bit modes: one row norm before the first block, five launches per block,
        blocks = 1 + 2 * depth * 5 + (1 if mel else 0)  # the deferred last SourceNorm
    else:
        blocks = 2 * depth * (7 + (1 if mel else 0))
    hidden = mask_layers if mel else mask_layers - 1
    model = 2 + blocks + (0 if mel else 1) + 1 + stems * (hidden + 1 + 1)  # split, blocks, final norm, cast, masks
    per_batch = 2 + model + 2 + 1          # gather + stft, model, istft (2), ola
    batches = -(-chunks // batch)
    return batches * per_batch + 1        # + finish


class Clocks:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index, self.samples, self._stop = index, [], threading.Event()
        self._proc = None

    def __enter__(self):
        q = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
        try:
            self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                           "--format=csv,noheader,nounits", "-lms", "200"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self._proc = None
        return self

    def _read(self):
        for line in self._proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self._proc:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 4 + i and s[4 + i].lower().startswith("active")})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.samples)}


def cpu_oracle_chunk(package: str, seconds_audio: float = CHUNK / SR):
    """Time the numpy oracle (f32) on one native chunk: gather → STFT → model → iSTFT → OLA."""
    from oracle import dsp, roformer, runtime
    model = roformer.Roformer(package, dtype=np.float32)
    planes = track(CHUNK / SR, 7)
    st = dsp.Stft(2048, HOP, dtype=np.float32)

    def one():
        t0 = time.perf_counter()
        spectra = [st.forward(p) for p in planes]
        masks = model.forward(runtime.pack_spectrum(spectra).astype(np.float32))
        y = runtime.apply_masks(spectra, masks, st, CHUNK, True)
        acc = dsp.Accumulator(2, CHUNK)
        acc.add(dsp.ChunkPlan(CHUNK, OVERLAP), 0, y[0])
        return time.perf_counter() - t0
    return model, one


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ensure_package(a.package, 0)
    _, one = cpu_oracle_chunk(a.package)
    advance = CHUNK / OVERLAP / SR  # new audio per native chunk (s)
    # One native chunk takes ~30 s on 16 cores: one warm-up and 3 timed samples (the median is
    # reported), so the arm ends within a few minutes whatever --steps / --warmup ask for (the
    # line reports the counts actually run).
    warmup, steps = 1, 3
    for _ in range(warmup):
        one()
    times = [one() for _ in range(steps)]
    t = float(np.median(times))
    value = advance / t
    cores = os.cpu_count()
    sample = (f"one native-context chunk (8 s window, {advance:.0f} s of new audio) of the Mel-Band "
              f"RoFormer per step through the numpy f32 port of the reference CPU path (not the "
              f"reference's own Burn CPU backend, which cannot be built here); median of {steps} "
              f"after {warmup} warm-up")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "×realtime",
        "n_gpus": a.gpus, "steps": steps, "warmup": warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "mel-band-roformer native context, CPU port"},
        "cpu_baseline": {"value": value, "unit": "×realtime", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "×realtime", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    import ctypes as C

    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from ancha_b200 import _native as N
    from ancha_b200.model import Roformer, separate_pcm

    ensure_package(a.package, rank if world == 1 else int(os.environ.get("LOCAL_RANK", "0")))
    model = Roformer(a.package, local, a.precision)
    planes = track(a.seconds, 1000 + rank)
    samples = planes.shape[1]
    chunks, length = plan_chunks(samples)
    d_planes = torch.from_numpy(planes).to(f"cuda:{local}")
    d_stems = torch.empty((model.stems, 2, samples), dtype=torch.float32, device=f"cuda:{local}")
    stream = torch.cuda.Stream()
    L = N.lib()

    def step():
        N.check(L.ancha_separate_device(model.handle, d_planes.data_ptr(), samples, CHUNK, OVERLAP,
                                        a.batch, d_stems.data_ptr(), C.c_void_p(stream.cuda_stream)))

    def barrier():
        if dist:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            step()
        N.check(L.ancha_separate_status(model.handle, C.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            ev0.record(stream)
            for _ in range(a.steps):
                step()
            ev1.record(stream)
            torch.cuda.synchronize()
        N.check(L.ancha_separate_status(model.handle, C.c_void_p(stream.cuda_stream)))
        barrier()
    ms = ev0.elapsed_time(ev1) / a.steps
    if a.pipeline_only:
        if rank == 0:
            print(json.dumps({"pipeline_only": True, "ms_per_step": ms, "chunks": chunks}), flush=True)
        model.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    t = torch.tensor([ms], device=f"cuda:{local}")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    audio_s = samples / SR
    value = world * audio_s / (ms / 1e3)

    # End to end through the public host API (pinned host PCM in, pinned host stems out).
    h_planes, h_stems = pinned(planes.shape), pinned((model.stems, 2, samples))
    h_planes[...] = planes
    for _ in range(2):
        separate_pcm([model], h_planes, CHUNK, OVERLAP, a.batch, out=h_stems)
    barrier()
    torch.cuda.synchronize()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for _ in range(a.steps):
        _, secs = separate_pcm([model], h_planes, CHUNK, OVERLAP, a.batch, out=h_stems)
    x1.record()
    torch.cuda.synchronize()
    e2e_s = x0.elapsed_time(x1) / 1e3 / a.steps  # CUDA events around the blocking host calls
    te = torch.tensor([e2e_s], device=f"cuda:{local}")
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    e2e = {"value": world * audio_s / e2e_s, "unit": "×realtime",
           "h2d_bytes_per_step": int(planes.nbytes), "d2h_bytes_per_step": int(model.stems * 2 * samples * 4)}

    # Dominant kernel alone: the FFN-in projection (rows = 60·801, 384 → 1536, GELU epilogue).
    hbm, tc_peak, tc_sus, peak_kind = peaks()
    from ancha_b200 import fused
    rows = 60 * 801
    x = torch.randn(rows, 384, device=f"cuda:{local}").to({"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[a.precision])
    w = (torch.randn(1536, 384, device=f"cuda:{local}") * 0.02).to(x.dtype)
    b = torch.zeros(1536, device=f"cuda:{local}")
    ep = fused.Epilogue(bias=b, gelu=True)
    for _ in range(3):
        fused.linear(x, w, ep, weight_layout=N.W_NK)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    e0.record()
    for _ in range(reps):
        fused.linear(x, w, ep, weight_layout=N.W_NK)
    e1.record()
    torch.cuda.synchronize()
    kms = e0.elapsed_time(e1) / reps
    flops = 2.0 * rows * 384 * 1536
    achieved = flops / (kms / 1e3) / 1e12
    roofline = {"kernel": "ffn_in linear (gemm, bias+GELU epilogue)", "bound": "tensor",
                "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s", "frac": achieved / tc_peak,
                "peak_kind": peak_kind,
                # DRAM bytes of one launch from an ncu capture of the same shape (cold cache);
                # profiles/gemm_tc_ffn_in_gelu.md has the command and the counters.
                "traffic": 134.10e6, "traffic_unit": "bytes per launch (dram read + write, ncu)",
                "algorithmic": f"2·{rows}·384·1536 flop per launch"}

    # Fused attention alone: time axis T = 801 / 1601 / 3201, band axis S = 60
    # (gated, in the model's packed layout), and the fp32 variant at T = 801.
    def time_attn(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    sweep = []
    for T in (801, 1601, 3201):
        q = torch.randn(60, T, 8, 64, device=f"cuda:{local}").to(x.dtype)
        ms_t = time_attn(lambda q=q: fused.attention(q, q, q))
        tf = 4.0 * 60 * 8 * T * T * 64 / (ms_t / 1e3) / 1e12
        sweep.append({"axis": "time", "shape": f"[B=60, H=8, T={T}, D=64]", "dtype": a.precision, "ms": ms_t,
                      "tflops": tf, "frac": tf / tc_peak})
    q = torch.randn(60, 801, 8, 64, device=f"cuda:{local}")
    ms_t = time_attn(lambda q=q: fused.attention(q, q, q), reps=3)
    tf = 4.0 * 60 * 8 * 801 * 801 * 64 / (ms_t / 1e3) / 1e12
    sweep.append({"axis": "time", "shape": "[B=60, H=8, T=801, D=64]",
                  "dtype": "f32 (tensor cores, three-plane bf16 split)", "ms": ms_t, "tflops": tf})
    packed = torch.randn(801, 60, 3 * 512 + 8, device=f"cuda:{local}").to(x.dtype)
    # Band axis in the model's layout is exercised by the model; standalone, [B=801, S=60] with
    # the gate columns of the packed projection.
    ms_t = time_attn(lambda: fused.gated_attention(packed, 8))
    moved = 801 * 60 * ((3 * 512 + 8) + 512) * 2
    sweep.append({"axis": "band", "shape": "[B=801, H=8, S=60, D=64] gated", "dtype": a.precision, "ms": ms_t,
                  "tflops": 4.0 * 801 * 8 * 60 * 60 * 64 / (ms_t / 1e3) / 1e12,
                  "gbs": moved / (ms_t / 1e3) / 1e9, "hbm_frac": moved / (ms_t / 1e3) / 1e9 / hbm})
    attention = dict(sweep[0], sweep=sweep[1:])

    strong = mel_track(model, local, world, rank, dist, a.precision)
    f32 = fp32_leg(a.package, local, world, rank, dist, planes, d_planes) if a.precision != "f32" else None

    c3 = None
    if not a.no_config3:
        c3 = config3(local, world, rank, dist)

    c4 = None
    if not a.no_config4:
        c4 = config4(local, world, rank, dist)

    c5 = None
    if not a.no_config5:
        c5 = config5(local, world, rank, dist)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        _, one = cpu_oracle_chunk(a.package)
        one()  # warm-up
        times = [one() for _ in range(3)]
        tcpu = float(np.median(times))
        cpu = {"value": (CHUNK / OVERLAP / SR) / tcpu, "unit": "×realtime", "cores": os.cpu_count(),
               "kind": "port",
               "sample": "one native-context chunk (8 s window, 2 s of new audio) through the numpy "
                         f"f32 port of the reference CPU path (not the reference's Burn CPU backend); "
                         f"median of 3 after 1 warm-up: {tcpu:.1f} s (samples "
                         f"{', '.join(f'{x:.1f}' for x in times)} s)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "×realtime", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": a.precision,
            "data": "synthetic (Gaussian sigma 0.1 stereo 44.1 kHz; seeded N(0,0.02) weights)",
            "config": {"workload": f"mel-band-roformer dim384 depth6 60 bands, native context "
                                   f"(chunk {CHUNK}, overlap {OVERLAP}), {a.seconds:.0f} s track "
                                   f"= {chunks} chunks per GPU",
                       "chunks_per_gpu": chunks, "batch_chunks": effective_batch(chunks, a.batch),
                       "l2": "working set > 126 MB L2 (no flush)", "parallelism": f"chunk-shard x{world}"},
            "clocks": clk.summary(), "e2e": e2e,
            "gpu_launches": launches_per_step(chunks, effective_batch(chunks, a.batch),
                                              fused=a.precision != "f32") * a.steps,
            "roofline": roofline, "attention": attention, "strong_track": strong, "fp32": f32, "config3": c3, "config4": c4,
            "config5": c5,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
