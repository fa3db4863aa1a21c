"""Benchmark of the voom_b200 weight-page decode path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1_rans|c2_vpack|c3_moe|c4_moe_ep|c5_nf12|c6_kv_paged]
                    [--tokens T] [--kernel-times] [--device-only]

Workloads: c1_rans (config 1), c2_vpack (config 2, the
default), c3_moe (config 3), c4_moe_ep (config 4, expert parallel), c6_kv_paged
(config 5, 65,536 KV pages), c5_nf12 (the NF12 sidecar, a next row).

A step is one pass of the hot path over one batch of synthetic input with
the shape of a BASELINE config (see `--workload`).  `value` is device
throughput with inputs resident in HBM (per-step CUDA events on the launching
stream, L2 flushed between steps, max over ranks); `e2e` is the same metric
through the public API with pinned host buffers and the host<->device copies
inside the timed region.  `--impl reference` times the CPU restatement of the
reference algorithm (the oracle port: the reference is pure Python and its
checkout does not travel to the GPU host) on all host cores.

Multi-GPU: one process per GPU (torchrun); pages/frames are independent
units, so every rank decodes its own copy of the workload with no collective
(weak scaling).
"""

from __future__ import annotations

import argparse
import json
import glob
import re
import os
import pickle
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo) and its logical cores."""
    name = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return f"{name}, {os.cpu_count()} logical cores"


def profiled_traffic(workload: str):
    """DRAM bytes per step of `workload` from the committed ncu summaries
    (a `traffic_bytes_per_step <workload>: N` line under profiles/), or None."""
    pat = re.compile(r"^traffic_bytes_per_step (\S+): (\d+)\s*$")
    for f in sorted(glob.glob(os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "*.md"))):
        with open(f) as fh:
            for line in fh:
                m = pat.match(line)
                if m and m.group(1) == workload:
                    return int(m.group(2)), os.path.join("profiles", os.path.basename(f))
    return None


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- workloads
class C1Rans:
    """Config 1: one 4096x4096 BF16 tensor (N(0,0.02), 0.1% outlier columns x50)
    as a VRN1 frame with the reference's default 1 MiB tiles; a step is one full
    cold decode of the frame (64 independent plane streams)."""

    name = "c1_rans_4096x4096"
    data = "synthetic (seeded numpy): BF16 N(0, 0.02), 0.1% of columns x50"
    metric = "BF16 weight-page decode GB/s (bit-exact)"
    unit = "GB/s"
    dtype = "u8"

    def __init__(self, device, rank: int):
        import torch

        from voom_b200 import _device, synthetic
        from voom_b200.formats import bf16_rans as R

        self.torch = torch
        self.R = R
        self.dev = device
        self.raw = synthetic.outlier_matrix(4096, 4096, seed=rank).tobytes()
        self.frame, self.stats = R.encode(self.raw, tile_bytes=1 << 20)
        self.plan = R.plan(self.frame)
        self.src = _device.upload(self.frame, device)
        self.tiles = _device.tensor_from_numpy(self.plan.tiles, device)
        self.out = torch.empty(len(self.raw), dtype=torch.uint8, device=device)
        self.status = torch.zeros(self.plan.info.n_tiles, dtype=torch.int32, device=device)
        self.n_tiles = int(self.plan.info.n_tiles)
        self.pinned_frame = _device.pinned_empty(len(self.frame))
        self.pinned_frame.numpy()[:] = np.frombuffer(self.frame, np.uint8)
        self.pinned_out = _device.pinned_empty(len(self.raw))
        self.units_per_step = len(self.raw)  # decoded bytes
        self.algo_bytes = len(self.frame) + len(self.raw)
        self.streams = 2 * int((self.plan.tiles["mode"] == 1).sum())

    def step_device(self, stream_ptr: int):
        from voom_b200._lib import check, load

        check(load().voom_rans_decode(self.src.data_ptr(), self.tiles.data_ptr(), self.n_tiles,
                                      self.out.data_ptr(), self.status.data_ptr(), None, None, 0, stream_ptr),
              "voom_rans_decode")

    def verify(self) -> bool:
        st = self.status.cpu().numpy()
        return bool((st == 0).all()) and self.out.cpu().numpy().tobytes() == self.raw

    def extra(self, stream, steps: int, flush) -> dict:
        """Warm decode of the same frame kept resident with a checkpoint index
        (every 256 symbols): all checkpoint segments run in parallel."""
        torch = self.torch
        page = self.R.RansPage(self.frame, device=self.dev, every=256)
        out = torch.empty(len(self.raw), dtype=torch.uint8, device=self.dev)
        st = torch.zeros(self.n_tiles, dtype=torch.int32, device=self.dev)
        page.decode_into(out, st, stream)
        torch.cuda.synchronize()
        ok = bool((st.cpu().numpy() == 0).all()) and out.cpu().numpy().tobytes() == self.raw
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            flush.fill_(3)
            a.record(stream)
            page.decode_into(out, st, stream)
            b.record(stream)
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        res = {"indexed_decode": {"value": round(len(self.raw) / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                                  "ms_per_step": round(ms, 5), "bit_exact": ok, "ckpt_every": 256,
                                  "index_bytes": int(page.ckpt.numel() * 4)}}
        # the same tensor framed with smaller tiles (more independent streams), cold decode
        from voom_b200 import _device
        from voom_b200._lib import check, load

        for tb, label in ((1 << 16, "tile_64KiB"), (1 << 14, "tile_16KiB")):
            frame, _ = self.R.encode(self.raw, tile_bytes=tb)
            plan = self.R.plan(frame)
            src = _device.upload(frame, self.dev)
            tiles = _device.tensor_from_numpy(plan.tiles, self.dev)
            nt = int(plan.info.n_tiles)
            st = torch.zeros(nt, dtype=torch.int32, device=self.dev)

            def run():
                check(load().voom_rans_decode(src.data_ptr(), tiles.data_ptr(), nt, out.data_ptr(), st.data_ptr(),
                                              None, None, 0, int(stream.cuda_stream)), "voom_rans_decode")

            run()
            torch.cuda.synchronize()
            ok = bool((st.cpu().numpy() == 0).all()) and out.cpu().numpy().tobytes() == self.raw
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for a, b in ev:
                flush.fill_(4)
                a.record(stream)
                run()
                b.record(stream)
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in ev) / steps
            res[label] = {"value": round(len(self.raw) / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                          "ms_per_step": round(ms, 5), "bit_exact": ok, "tiles": nt,
                          "frame_bytes": len(frame), "ratio": round(len(self.raw) / len(frame), 4)}
        return res

    def step_e2e(self):
        out = self.R.decode_device(self.pinned_frame, device=self.dev)
        self.pinned_out.copy_(out, non_blocking=True)
        return len(self.frame) + 8 * self.n_tiles, len(self.raw) + 4 * self.n_tiles

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """Oracle (C restatement of bf16_rans.decode) on whole frames, one frame
        per thread, repeated until `budget_s` of wall time."""
        from concurrent.futures import ThreadPoolExecutor

        from oracle import rans as orans

        assert orans.decode(self.frame) == self.raw
        done = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while time.perf_counter() - t0 < budget_s:
                list(pool.map(lambda _: orans.decode(self.frame), range(threads)))
                done += threads
        dt = time.perf_counter() - t0
        return {"value": done * len(self.raw) / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{done} full C1 frame decodes ({len(self.raw)} B each) by the C oracle on {threads} "
                          f"thread(s), {dt:.1f} s"}

    def config(self) -> dict:
        return {"workload": self.name, "tile_bytes": 1 << 20, "tiles": self.n_tiles,
                "independent_streams": self.streams, "frame_bytes": len(self.frame),
                "raw_bytes": len(self.raw), "ratio": round(len(self.raw) / len(self.frame), 4),
                "l2": "flushed between steps (512 MiB write)"}


def lpt_partition(sizes, world: int) -> list[list[int]]:
    """Longest-processing-time split of items over `world` bins by size:
    items by descending size (ties by index), each to the least-filled bin."""
    bins = [[] for _ in range(world)]
    fill = [0] * world
    for k in sorted(range(len(sizes)), key=lambda k: (-sizes[k], k)):
        r = min(range(world), key=lambda b: (fill[b], b))
        bins[r].append(k)
        fill[r] += sizes[k]
    return [sorted(b) for b in bins]


class C2Vpack:
    """Config 2: the vpack2 archive of a random-init SmolLM2-135M-shaped
    checkpoint (30 layers, hidden 576, intermediate 1536, 9/3 heads x 64,
    vocab 49152, every tensor BF16 N(0, 0.02)), packed as the reference packs
    it (hi plane zstd level 1 + raw lo plane per tensor, access order).  A step
    decodes every body of the archive back to BF16 bytes.  With N ranks the
    bodies are split by compressed bytes (LPT); each rank decodes its share in
    one batched GPU decode and an NCCL all-gather leaves the whole decoded
    archive on every rank (the replicated-weights case)."""

    name = "c2_vpack2_smollm2_135m"
    data = "synthetic (seeded numpy): random-init SmolLM2-135M shapes, every tensor BF16 N(0, 0.02)"
    metric = "BF16 weight-page decode GB/s (bit-exact)"
    unit = "GB/s"
    dtype = "u8"

    def __init__(self, device, rank: int, layers: int = 30, world: int = 1):
        import torch
        from concurrent.futures import ThreadPoolExecutor

        from voom_b200 import _device, synthetic
        from voom_b200.formats import packed, packed2, zstd_gpu

        self.torch = torch
        self.dev = device
        self.packed = packed
        self.rank, self.world = rank, world
        specs = synthetic.smollm2_tensors(dict(synthetic.SMOLLM2_135M, layers=layers))
        if layers != 30:
            self.name = f"c2_vpack2_smollm2_135m_{layers}layers"
        import zlib

        def make(spec):
            name, shape = spec
            bits = synthetic.bf16_normal(shape, 0.02, zlib.crc32(name.encode()))
            head, body = packed.body_for("BF16", bits.view(np.uint8))
            return name, {"dtype": "BF16", "shape": list(shape), **head}, body, bits

        threads = max(2, (os.cpu_count() or 8) // max(1, world))
        with ThreadPoolExecutor(max_workers=threads) as pool:
            items = list(pool.map(make, specs))
        order = packed2.access_order([n for n, _, _, _ in items])
        by = {n: (h, b, r) for n, h, b, r in items}
        self.all_names = order
        self.raws = {n: by[n][2] for n in order}
        self.raw_bytes = sum(r.nbytes for r in self.raws.values())
        self.archive_bytes = sum(len(by[n][1]) for n in order)
        self.parts = lpt_partition([len(by[n][1]) for n in order], world)
        mine = [order[k] for k in self.parts[rank]]
        self.names = mine
        self.heads = [by[n][0] for n in mine]
        bodies = [by[n][1] for n in mine]
        self.offs, self.lens = [], []
        pos = 0
        for b in bodies:
            self.offs.append(pos)
            self.lens.append(len(b))
            pos += len(b)
        self.archive = np.frombuffer(b"".join(bodies), np.uint8)
        self.pinned = _device.pinned_empty(self.archive.size)
        self.pinned.numpy()[:] = self.archive
        self.src = _device.upload(self.archive, device)
        # each rank's decoded share in a slot of `cap` bytes of the gathered buffer
        self.layout = {}
        cap = 0
        for r, part in enumerate(self.parts):
            dst = 0
            for k in part:
                n = self.raws[order[k]].nbytes
                self.layout[order[k]] = (r, dst, n)
                dst += (n + 255) // 256 * 256
            cap = max(cap, dst)
        self.cap = cap
        jobs, self.spans = [], []
        for h, o, ln, name in zip(self.heads, self.offs, self.lens, mine):
            _, d, _ = self.layout[name]
            job, n = packed.body_job(h, o, ln, d)
            jobs.append(job)
            self.spans.append((d, n))
        self.plan = zstd_gpu.ZstdPlan(self.archive, np.concatenate(jobs))
        self.batch = zstd_gpu.ZstdBatch(self.plan, device)
        self.out = torch.zeros(cap, dtype=torch.uint8, device=device)
        self.full = torch.zeros(cap * world, dtype=torch.uint8, device=device) if world > 1 else self.out
        self.units_per_step = self.raw_bytes  # the whole archive decoded (and replicated) per step
        self.local_raw = sum(self.raws[n].nbytes for n in mine)
        self.algo_bytes = self.archive.size + self.local_raw  # this rank's decode
        self.gather_bytes = cap * (world - 1) if world > 1 else 0
        self.n_blocks = int(self.plan.info.n_blocks)
        self.launches_per_step = 13  # K0 K1 K1b K2 K3 K5 5xK4 patch K6 (+ the NCCL all-gather with N > 1)
        self.scaling = "strong" if world > 1 else "weak"
        self.replicated_units = True  # value = the one archive's bytes, not x N

    def _gather(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.full, self.out)

    def step_device(self, stream_ptr: int):
        self.batch.run(self.src, self.out, self.torch.cuda.current_stream(self.dev))
        self._mark = self.torch.cuda.Event(enable_timing=True)
        self._mark.record()
        self._gather()

    def verify(self) -> bool:
        if self.batch.job_status().any():
            return False
        got = self.full.cpu().numpy()
        for n, (r, d, ln) in self.layout.items():
            o = r * self.cap + d if self.world > 1 else d
            if not np.array_equal(got[o:o + ln], self.raws[n].reshape(-1).view(np.uint8)):
                return False
        return True

    def step_e2e(self):
        out, spans = self.packed.decode_bodies(self.heads, self.pinned, self.offs, self.lens,
                                               device=self.dev, src_dev=None)
        if self.world > 1:
            import torch.distributed as dist

            part = self.out
            for (d, n), (d2, _) in zip(spans, self.spans):
                part[d2:d2 + n].copy_(out[d:d + n])
            dist.all_gather_into_tensor(self.full, part)
        return self.archive.size, 4 * len(self.heads)

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """The reference decode leg (decode_body: libzstd + numpy interleave per
        body) over this rank's bodies, spread over `threads` host threads,
        repeated until `budget_s` of wall time."""
        from concurrent.futures import ThreadPoolExecutor

        from oracle import vpack as ov

        arch = self.archive
        items = list(zip(self.heads, self.offs, self.lens))
        ok = ov.decode_body(items[1][0], arch[items[1][1]:items[1][1] + items[1][2]])
        assert np.array_equal(ok, self.raws[self.names[1]].reshape(-1).view(np.uint8))
        done = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while time.perf_counter() - t0 < budget_s:
                for r in pool.map(lambda it: ov.decode_body(it[0], arch[it[1]:it[1] + it[2]]).size, items):
                    done += r
        dt = time.perf_counter() - t0
        return {"value": done / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "cpu_model": cpu_model(),
                "sample": f"{done / self.local_raw:.2f} passes over the {len(items)}-body archive "
                          f"({self.local_raw} B decoded per pass) with decode_body restated (libzstd + numpy) "
                          f"on {threads} thread(s), {dt:.1f} s"}

    def repack_leg(self, threads: int, reps: int = 3) -> dict:
        """The GPU repack of this archive's tensors (packed.bodies_gpu: byte
        planes split on the device, hi planes encoded by the GPU zstd encoder)
        against host zstd level 1 (the reference's pack call) on `threads`
        threads: raw tensor bytes per second, and the bodies' total size."""
        torch = self.torch
        from concurrent.futures import ThreadPoolExecutor

        from voom_b200.formats import packed, zstd_gpu, zstd_host

        names = self.names
        dev_t = [torch.from_numpy(self.raws[n].reshape(-1).view(np.uint8).copy()).to(self.dev) for n in names]
        raw_bytes = sum(int(t.numel()) for t in dev_t)
        items = [("BF16", t) for t in dev_t]
        bodies = packed.bodies_gpu(items)  # warm-up (and the size)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            bodies = packed.bodies_gpu(items)
        e2e_s = (time.perf_counter() - t0) / reps
        gpu_bytes = sum(len(b) for _, b in bodies)
        # device encode alone: the hi planes at 16-byte offsets, one EncodePlan, CUDA events
        offs, lens, pos = [], [], 0
        for t in dev_t:
            offs.append(pos)
            lens.append(int(t.numel()) // 2)
            pos += (int(t.numel()) // 2 + 15) // 16 * 16
        hi = torch.empty(pos, dtype=torch.uint8, device=self.dev)
        for o, n, t in zip(offs, lens, dev_t):
            hi[o:o + n].copy_(t[1::2])
        plan = zstd_gpu.EncodePlan(offs, lens, self.dev)
        plan.run(hi)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            plan.run(hi)
        b.record()
        torch.cuda.synchronize()
        dev_ms = a.elapsed_time(b) / reps
        # host: zstd level 1 of the hi planes (+ the lo plane copy), bounded sample
        host_items = [self.raws[n].reshape(-1).view(np.uint8) for n in names]

        def one(arr):
            return len(zstd_host.compress(np.ascontiguousarray(arr[1::2]), 1)) + arr.size // 2

        done = host_bytes = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while time.perf_counter() - t0 < 2.0 or done == 0:
                host_bytes = sum(pool.map(one, host_items))
                done += 1
        host_s = (time.perf_counter() - t0) / done
        del dev_t, hi
        return {"metric": "vpack repack GB/s (raw tensor bytes in, bodies out)", "unit": "GB/s",
                "device_encode": round(raw_bytes / (dev_ms * 1e-3) / 1e9, 3),
                "device_encode_ms": round(dev_ms, 4),
                "e2e": round(raw_bytes / e2e_s / 1e9, 3),
                "e2e_note": "packed.bodies_gpu: plane split and encode on the device, bodies in host memory",
                "host_libzstd_level1": round(raw_bytes / host_s / 1e9, 3), "host_threads": threads,
                "body_bytes_gpu": int(gpu_bytes), "body_bytes_host_level1": int(host_bytes),
                "tensors": len(names), "raw_bytes": int(raw_bytes)}

    def config(self) -> dict:
        return {"workload": self.name, "tensors": len(self.all_names), "zstd_blocks_this_rank": self.n_blocks,
                "archive_bytes": int(self.archive_bytes), "raw_bytes": int(self.raw_bytes),
                "ratio": round(self.raw_bytes / self.archive_bytes, 4), "zstd_level": 1,
                "parallelism": (f"partition x{self.world}: bodies split by compressed bytes (LPT), NCCL "
                                f"all-gather of the decoded bodies inside the step" if self.world > 1 else "single"),
                "bodies_this_rank": len(self.names), "archive_bytes_this_rank": int(self.archive.size),
                "l2": "flushed between steps (512 MiB write); inputs 184 MB + output 269 MB exceed L2"}


class C3Moe:
    """Config 3: MoE expert streaming decode step -- hidden 2048, 128 experts
    with SwiGLU gate/up 2048->768 and down 768->2048 (BF16 N(0, 0.02)) kept as
    rANS-coded pages in HBM, top-8 softmax routing from a random router, 48
    layers, fused decode + GEMV.  A step runs all 48 layers for T tokens
    (`--tokens`, 1 or 8); the metric is tokens per second.  The 48 layers
    share one set of 128 experts' pages (each layer has its own router), so
    the per-layer decode work is the configuration's while the page set is
    128 x 9 MiB instead of 48 x 128 x 9 MiB."""

    metric = "fused expert GEMV tok/s (48-layer MoE decode step)"
    data = "synthetic (seeded torch): experts BF16 N(0, 0.02), router N(0, 1), tokens N(0, 1)"
    unit = "tok/s"
    dtype = "bf16"

    def __init__(self, device, rank: int, tokens: int = 1, layers: int = 48, store=None):
        import torch

        from voom_b200 import synthetic
        from voom_b200.runtime import moe

        self.torch = torch
        self.dev = device
        self.T = tokens
        self.L = layers
        self.name = f"c3_moe_h2048_e128_i768_top8_T{tokens}_L{layers}"
        E, H, I = 128, 2048, 768
        g = torch.Generator().manual_seed(4242)

        def weight(e, j):
            shape = (I, H) if j < 2 else (H, I)
            return lambda: synthetic.bf16_normal(shape, 0.02, 90_000 + 3 * e + j)

        experts = [tuple(weight(e, j) for j in range(3)) for e in range(E)]
        if store is None:
            store = moe.ExpertStore(experts, device, threads=max(2, os.cpu_count() or 8))
        self.store = store
        self.layers = []
        for _ in range(layers):
            wr = torch.randn((E, H), generator=g).to(torch.bfloat16).to(device)
            # post-attention RMSNorm weight of the layer (keeps the 48-layer chain finite)
            nw = (1.0 + 0.05 * torch.randn(H, generator=g)).to(torch.bfloat16).to(device)
            self.layers.append(moe.MoeLayer(self.store, wr, nw, top_k=8, norm_topk=True))
        self.x0 = torch.randn((tokens, H), generator=g).to(torch.bfloat16).to(device)
        self.bufs = [torch.empty_like(self.x0) for _ in range(2)]
        self.x_host = torch.randn((tokens, H), generator=g).to(torch.bfloat16).pin_memory()
        self.y_host = torch.empty((tokens, H), dtype=torch.bfloat16).pin_memory()
        self.units_per_step = tokens
        per_expert = self.store.compressed_bytes / E
        self.routed = None
        self.per_expert_bytes = per_expert
        self.algo_bytes = None  # set after a routing pass (distinct experts per layer)
        self.launches_per_step = 7 * layers  # router logits, top-k, plan, gate/up, act, down, combine
        self.experts_raw = experts
        # the 48-layer step as one CUDA graph (bit-identical to the eager layers)
        self.graph = moe.MoeStepGraph(self.layers, tokens, H, device)
        self.graph.x.copy_(self.x0)

    def _run(self, x, stream):
        a, b = self.bufs
        cur = x
        for i, layer in enumerate(self.layers):
            out = a if i % 2 == 0 else b
            layer(cur, out=out, stream=stream)
            cur = out
        return cur

    def step_device(self, stream_ptr: int):
        self.graph.replay()
        if self.algo_bytes is None:
            self.torch.cuda.synchronize()
            # distinct routed experts per layer from the route tables (T*k <= 64)
            import ctypes
            n = 0
            for layer in self.layers:
                n += int(layer.scratch(self.T)[:4].view(self.torch.int32).item())
            self.distinct = n
            self.algo_bytes = int(n * self.per_expert_bytes + 2 * 2 * self.T * 2048 * self.L)

    def verify(self) -> bool:
        from oracle import moe as om

        torch = self.torch
        layer = self.layers[0]
        out = layer(self.x0, residual=False).cpu()
        raw = self.experts_raw

        class Lazy:  # the oracle reads only the routed experts
            def __getitem__(self, e):
                return tuple(torch.from_numpy(w().view(np.int16)).view(torch.bfloat16) for w in raw[e])

        ex = Lazy()
        ref = om.moe_layer(self.x0.cpu(), layer.router_w.cpu(), layer.norm_w.cpu(), ex, 8, True, residual=False)
        ok = om.rel_l2(out, ref) < 1e-2 and all(int(l.status.item()) == 0 for l in self.layers)
        # the replayed graph computes exactly the eager 48-layer stack
        eager = self._run(self.x0, torch.cuda.current_stream(self.dev)).clone()
        ok = ok and torch.equal(self.graph.replay(), eager)
        return ok

    def step_e2e(self):
        x = self.x_host.to(self.dev, non_blocking=True)
        y = self.graph.step(x)
        self.y_host.copy_(y, non_blocking=True)
        return self.T * 2048 * 2, self.T * 2048 * 2

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """The reference's layer math restated in torch-CPU with rANS page
        decode by the C oracle (one layer per sample unit)."""
        from oracle import moe as om
        from oracle import rans as orans

        torch = self.torch
        torch.set_num_threads(threads)
        layer = self.layers[0]
        wr = layer.router_w.cpu()
        nw = layer.norm_w.cpu()
        x = self.x0.cpu()
        frames = [[bytes(p.page.src[: p.frame_bytes].cpu().numpy()) for p in trip] for trip in self.store.pages]
        done = 0
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < budget_s or done == 0:
            h = om.rms_norm(x, nw, 1e-6)
            idx, _ = om.route(h, wr, 8, True)
            needed = sorted({int(e) for e in idx.flatten()})
            ex = {}
            for e in needed:  # decode the routed experts' pages (the reference decodes on fetch)
                ws = []
                for fr, (rows, cols) in zip(frames[e], ((768, 2048), (768, 2048), (2048, 768))):
                    raw = np.frombuffer(orans.decode(fr), np.int16).reshape(rows, cols)
                    ws.append(torch.from_numpy(raw.copy()).view(torch.bfloat16))
                ex[e] = tuple(ws)
            om.moe_layer(x, wr, nw, ex, 8, True)
            done += 1
        dt = time.perf_counter() - t0
        tok_s = self.T / (dt / done * self.L)
        return {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{done} layer(s) of T={self.T}: C-oracle rANS decode of the routed experts + torch-CPU "
                          f"layer math on {threads} thread(s), {dt:.1f} s, scaled to {self.L} layers"}

    def config(self) -> dict:
        return {"workload": self.name, "tokens": self.T, "layers": self.L, "experts": 128, "hidden": 2048,
                "intermediate": 768, "top_k": 8, "page_bytes_compressed": int(self.store.compressed_bytes),
                "page_bytes_raw": int(self.store.raw_bytes),
                "ratio": round(self.store.raw_bytes / self.store.compressed_bytes, 4),
                "distinct_experts_per_step": getattr(self, "distinct", None),
                "l2": "flushed between steps (512 MiB write); 128 experts' pages (~770 MB) exceed L2"}


class C4MoeEP:
    """Config 4: the large-MoE layer sharded over the ranks -- hidden 6144, 160
    distinct experts with intermediate 2048 (BF16 N(0, 0.015)), each
    projection a VRN1 frame of 2 MiB pages (12 per projection) with a
    checkpoint index, top-8 softmax routing whose expert popularity follows
    Zipf(1.1) (router logits biased by c log p over a seeded permutation of
    ranks; top-8 then approximates drawing 8 distinct experts in proportion to
    the popularity), T tokens per step.  Expert parallel: every rank routes all tokens
    and runs the fused decode + SwiGLU of the experts it owns (placed by LPT over
    the expected decode cost of the T values timed; with N > 1 the 8 hottest are
    held by every rank and each routed one is computed by its least loaded
    holder); the token-major route rows are reduce-scattered over tokens, each
    rank combines its tokens, and an all-gather shares the combined rows.  A step runs `layers` layers (one router
    each) over the same expert set, the configuration's single layer; the
    metric is tokens per second through one layer (T x layers / step time)."""

    metric = "fused expert GEMV tok/s through one MoE layer (expert parallel)"
    unit = "tok/s"
    dtype = "bf16"
    data = ("synthetic (seeded numpy/torch): 160 distinct experts BF16 N(0, 0.015) in 2 MiB rANS pages, "
            "router N(0, 0.02) + a log Zipf(1.1) popularity bias, tokens N(0, 1)")
    E, H, I, K = 160, 6144, 2048, 8
    PAGE = 2 << 20
    REPLICATED = 8  # hottest experts held by every rank when N > 1

    def __init__(self, device, rank: int, world: int = 1, tokens=(1, 8, 64), layers: int = 4):
        import torch

        from voom_b200 import synthetic
        from voom_b200.runtime import moe

        self.torch = torch
        self.dev = device
        self.rank, self.world = rank, world
        self.L = layers
        E, H, I = self.E, self.H, self.I
        self.pop = moe.zipf_popularity(E, 1.1, seed=11)
        gr = torch.Generator().manual_seed(4242)  # identical routers on every rank
        logp = torch.from_numpy(np.log(self.pop)).float()
        # router logits of unit-variance tokens have noise sigma = 0.02 sqrt(H);
        # a bias of (sigma / 1.28) log p sets that noise against log p like a
        # standard Gumbel (std 1.28), so top-8 approximates drawing 8 distinct
        # experts in proportion to the Zipf popularity (Plackett-Luce)
        self.bias_scale = 0.02 * float(np.sqrt(H)) / 1.28
        self.bias = (self.bias_scale * logp).to(device)
        self.routers = []
        for _ in range(layers):
            wr = (torch.randn((E, H), generator=gr) * 0.02).to(torch.bfloat16)
            nw = (1.0 + 0.05 * torch.randn(H, generator=gr)).to(torch.bfloat16)
            self.routers.append((wr, nw))
        self.cost = self._expected_cost(tokens)
        # with N > 1 the REPLICATED hottest experts are held by every rank and
        # assigned per step to the least loaded holder; the rest are placed LPT
        self.replicated = [int(e) for e in np.argsort(-self.cost, kind="stable")[:self.REPLICATED]] if world > 1 else []
        rest = np.array([e for e in range(E) if e not in self.replicated])
        self.placement = [sorted(int(rest[i]) for i in b) for b in moe.place_experts(self.cost[rest], world)]
        self.holders = moe.holders_for(self.placement, E, self.replicated)
        self.owned = sorted(set(self.placement[rank]) | set(self.replicated))

        def weight(e, j):
            shape = (I, H) if j < 2 else (H, I)
            return lambda: synthetic.bf16_normal(shape, 0.015, 50_000 + 3 * e + j)

        table = [None] * E
        for e in self.owned:
            table[e] = tuple(weight(e, j) for j in range(3))
        threads = max(2, (os.cpu_count() or 8) // max(1, world))
        t0 = time.perf_counter()
        self.store = moe.ExpertStore(table, device, tile_bytes=self.PAGE, threads=threads)
        self.setup_s = time.perf_counter() - t0
        self.expert_bytes = {e: sum(p.frame_bytes for p in self.store.pages[e]) for e in self.owned}
        self.layers = [moe.ExpertParallelMoeLayer(self.store, wr.to(device), nw.to(device), top_k=self.K,
                                                  router_bias=self.bias, holders=self.holders, rank=rank,
                                                  world=world) for wr, nw in self.routers]

    def _expected_cost(self, tokens) -> np.ndarray:
        """Expected page decodes per expert and step, averaged over the timed T
        values: 1 - (1 - q_e)^T with q_e the probability that a token routes to
        expert e, estimated with the routers on 2048 random tokens (host)."""
        torch = self.torch
        from oracle import moe as om

        g = torch.Generator().manual_seed(99)
        x = torch.randn((2048, self.H), generator=g).to(torch.bfloat16)
        q = np.zeros(self.E)
        for wr, nw in self.routers:
            h = om.rms_norm(x, nw, 1e-6)
            idx, _ = om.route(h, wr, self.K, True, bias=self.bias.cpu())
            q += np.bincount(idx.reshape(-1).numpy(), minlength=self.E) / x.shape[0]
        q = np.clip(q / len(self.routers), 0.0, 1.0)
        return np.mean([1.0 - (1.0 - q) ** T for T in tokens], axis=0)

    def for_tokens(self, T: int) -> "C4Step":
        return C4Step(self, T)

    def config(self) -> dict:
        raw = self.store.raw_bytes
        return {"workload": f"c4_moe_ep_h6144_e160_i2048_top8_x{self.world}", "experts": self.E,
                "distinct_experts": self.E, "hidden": self.H, "intermediate": self.I, "top_k": self.K,
                "page_bytes": self.PAGE, "layers_per_step": self.L,
                "layer_note": "one expert set (config 4's single layer) under `layers_per_step` routers",
                "local_experts": len(self.owned), "local_page_bytes_compressed": int(self.store.compressed_bytes),
                "local_page_bytes_raw": int(raw), "ratio": round(raw / max(1, self.store.compressed_bytes), 4),
                "popularity": f"Zipf(1.1) over a seeded permutation, router bias {self.bias_scale:.3f} log p "
                              "(top-8 ~ 8 distinct draws in proportion to the popularity)",
                "placement": ("LPT over expected page decodes per step (mean over the timed T)" +
                              (f"; the {len(self.replicated)} hottest experts held by every rank, each routed one "
                               "computed by its least loaded holder (rule evaluated on the device)"
                               if self.replicated else "")),
                "experts_per_rank": [len(b) + len(self.replicated) for b in self.placement],
                "replicated_experts": len(self.replicated),
                "combine": ("route rows in token-major order (zero where another rank computes them), NCCL "
                            "reduce-scatter over tokens, ordered BF16 combine of each rank's tokens, NCCL "
                            "all-gather of the combined rows" if self.world > 1 else
                            "ordered BF16 combine (one GPU)"),
                "page_build_s": round(self.setup_s, 2),
                "l2": "flushed between steps (512 MiB write); the page set exceeds L2"}


class C4Step:
    """One T of the config-4 sweep over a built C4MoeEP."""

    unit = "tok/s"

    def __init__(self, c4: C4MoeEP, T: int):
        torch = c4.torch
        self.c4, self.T, self.torch = c4, T, torch
        gx = torch.Generator().manual_seed(7000 + T)  # identical tokens on every rank
        x = torch.randn((T, c4.H), generator=gx).to(torch.bfloat16)
        self.x0 = x.to(c4.dev)
        self.bufs = [torch.empty_like(self.x0) for _ in range(2)]
        self.x_host = x.pin_memory()
        self.y_host = torch.empty_like(self.x_host).pin_memory()
        self.units_per_step = T * c4.L
        self.algo_bytes = None
        # router logits, top-k, plan, 2x gate/up, act, 2x down, combine (+ owners and token-major rows with N > 1)
        self.launches_per_step = (11 if c4.world > 1 else 9) * c4.L
        self.nccl_ms = 0.0

    def _run(self, x, timing: bool = False):
        cur = x
        ev = []
        for i, layer in enumerate(self.c4.layers):
            out = self.bufs[i % 2]
            if timing and self.c4.world > 1:
                import torch.distributed as dist

                ab = [self.torch.cuda.Event(enable_timing=True) for _ in range(4)]
                y = layer.experts(cur)
                _, _, shard, part, full = layer.buffers(self.T)
                ts = layer.t_pad(self.T) // self.c4.world
                ab[0].record()
                dist.reduce_scatter_tensor(shard, y)
                ab[1].record()
                layer.combine(cur, shard, part, self.c4.rank * ts, ts)
                ab[2].record()
                dist.all_gather_into_tensor(full, part)
                ab[3].record()
                out.copy_(full[:self.T])
                ev += [(ab[0], ab[1]), (ab[2], ab[3])]
            else:
                layer(cur, out=out)
            cur = out
        return cur, ev

    def step_device(self, stream_ptr: int):
        _, ev = self._run(self.x0, timing=True)
        self._ev = ev
        if self.algo_bytes is None:
            self._count_bytes()

    def collective_ms(self) -> float:
        self.torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in getattr(self, "_ev", []))

    def _count_bytes(self):
        """Compressed bytes of this rank's routed experts over the step's layers
        (read from the route tables) + the activations in and out."""
        torch = self.torch
        torch.cuda.synchronize()
        from voom_b200.runtime import moe

        n_local, byt, distinct = 0, 0, []
        for layer in self.c4.layers:
            s = layer.buffers(self.T)[0]
            words = s[:4 * (4 + 2 * 513)].view(torch.int32).cpu().numpy()
            nu = int(words[0])
            ex = [int(e) for e in words[4:4 + nu]]
            ntok = [int(n) for n in words[4 + 513:4 + 513 + nu]]
            distinct.append(nu)
            owner = moe.assign_owners(ex, ntok, self.c4.holders, self.c4.world)  # the device's rule
            mine = [e for e, o in zip(ex, owner) if o == self.c4.rank]
            n_local += len(mine)
            byt += sum(self.c4.expert_bytes[e] for e in mine)
        self.local_routed = n_local
        self.distinct_per_layer = distinct
        self.algo_bytes = int(byt + 2 * 2 * self.T * self.c4.H * self.c4.L)

    def verify(self) -> bool:
        for layer in self.c4.layers:
            layer.check_status()
        return True

    def step_e2e(self):
        x = self.x_host.to(self.c4.dev, non_blocking=True)
        y, _ = self._run(x)
        self.y_host.copy_(y, non_blocking=True)
        return self.T * self.c4.H * 2, self.T * self.c4.H * 2

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """The reference's CPU path for one layer at this T: decode the routed
        experts' rANS pages with the C oracle (one page per thread) and run the
        layer math in torch-CPU (the oracle restatement of run_moe_mlp); rank 0
        of a single-GPU run holds every expert."""
        torch = self.torch
        from concurrent.futures import ThreadPoolExecutor

        from oracle import moe as om
        from oracle import rans as orans

        torch.set_num_threads(threads)
        wr, nw = self.c4.routers[0]
        x = self.x0.cpu()
        bias = self.c4.bias.cpu()
        pages = self.c4.store.pages
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or done == 0:
            h = om.rms_norm(x, nw, 1e-6)
            idx, _ = om.route(h, wr, self.c4.K, True, bias=bias)
            need = sorted({int(e) for e in idx.flatten()})
            jobs = [(e, j) for e in need for j in range(3)]

            def dec(item):
                p = pages[item[0]][item[1]]
                raw = np.frombuffer(orans.decode(bytes(p.page.src[:p.frame_bytes].cpu().numpy())), np.int16)
                return item, torch.from_numpy(raw.reshape(p.rows, p.cols).copy()).view(torch.bfloat16)

            with ThreadPoolExecutor(max_workers=threads) as pool:
                got = dict(pool.map(dec, jobs))
            ex = {e: tuple(got[(e, j)] for j in range(3)) for e in need}
            om.moe_layer(x, wr, nw, ex, self.c4.K, True, bias=bias)
            done += 1
        dt = time.perf_counter() - t0
        return {"value": self.T * done / dt, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{done} layer(s) of T={self.T}: C-oracle rANS decode of the routed experts' pages "
                          f"({threads} threads) + torch-CPU layer math, {dt:.1f} s"}


class C5Nf12:
    """BF16 NF12 exact sidecar (the reference's next fused decode -> GEMV
    format): the seven projections of one Llama-3-8B-shaped decoder layer
    (q 4096x4096, k/v 1024x4096, o 4096x4096, gate/up 14336x4096, down
    4096x14336; BF16 N(0, 0.02) with 0.01% outliers that need patches) kept as
    one NF12 layer stream in HBM.  A step multiplies `--tokens` activation rows
    by all seven weights through the fused decode + small-M linear; the metric
    is BF16-equivalent weight bytes streamed per second."""

    data = "synthetic (seeded numpy): BF16 N(0, 0.02), 0.01% outliers N(0, 8)"
    metric = "NF12 fused decode + linear, BF16-equivalent weight GB/s"
    unit = "GB/s"
    dtype = "fp32-acc bf16"
    SHAPES = (("self_attn.q_proj", 4096, 4096), ("self_attn.k_proj", 1024, 4096), ("self_attn.v_proj", 1024, 4096),
              ("self_attn.o_proj", 4096, 4096), ("mlp.gate_proj", 14336, 4096), ("mlp.up_proj", 14336, 4096),
              ("mlp.down_proj", 4096, 14336))

    def __init__(self, device, rank: int, tokens: int = 1):
        import torch

        from voom_b200 import _device, synthetic
        from voom_b200.formats import nf12

        self.torch = torch
        self.nf12 = nf12
        self.dev = device
        self.M = tokens
        self.name = f"c5_nf12_llama8b_layer_M{tokens}"
        tensors = []
        for i, (name, n, k) in enumerate(self.SHAPES):
            bits = synthetic.bf16_normal((n, k), 0.02, 500 + i + 31 * rank).reshape(-1).copy()
            idx = np.random.default_rng(600 + i).choice(bits.size, bits.size // 10000, replace=False)
            bits[idx] = synthetic.bf16_normal((idx.size,), 8.0, 700 + i).reshape(-1)
            tensors.append((f"model.layers.0.{name}.weight", bits, (n, k)))
        self.payload, self.entry = nf12.build_layer(tensors)
        self.raw_bytes = sum(b.size * 2 for _, b, _ in tensors)
        self.enc = _device.upload(np.frombuffer(self.payload, np.uint8), device)
        self.specs = self.entry["tensors"]
        lib = self.lib = __import__("voom_b200._lib", fromlist=["load"]).load()
        g = torch.Generator().manual_seed(77 + rank)
        self.x = torch.randn((tokens, 4096), generator=g).to(torch.bfloat16).to(device)
        self.x14 = torch.randn((tokens, 14336), generator=g).to(torch.bfloat16).to(device)
        self.outs, self.scratch = [], []
        self.launches_per_step = 0
        for sp in self.specs:
            n, k = sp["shape"]
            need = int(lib.voom_nf12_linear_scratch_bytes(tokens, k, n))
            self.scratch.append((torch.empty(max(need, 1), dtype=torch.uint8, device=device), need))
            self.outs.append(torch.empty((tokens, n), dtype=torch.bfloat16, device=device))
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.launches_per_step = 2  # the batched fused linear (+ the reduce of split K ranges)
        self.units_per_step = self.raw_bytes
        self.algo_bytes = len(self.payload) + sum(2 * tokens * (sp["shape"][0] + sp["shape"][1]) for sp in self.specs)
        self.tensors = [nf12.NF12Tensor(self.enc, self.entry, sp) for sp in self.specs]
        self.x_host = torch.empty((tokens, 4096), dtype=torch.bfloat16).pin_memory()
        self.x_host.copy_(self.x.cpu())
        self.x14_host = torch.empty((tokens, 14336), dtype=torch.bfloat16).pin_memory()
        self.x14_host.copy_(self.x14.cpu())
        self.out_host = [torch.empty((tokens, sp["shape"][0]), dtype=torch.bfloat16).pin_memory()
                         for sp in self.specs]

    def _x(self, sp, x, x14):
        return x14 if sp["shape"][1] == 14336 else x

    def _tasks(self, x, x14, outs):
        import ctypes

        from voom_b200.formats.nf12 import LinearTask

        arr = (LinearTask * len(self.specs))()
        for i, (sp, out) in enumerate(zip(self.specs, outs)):
            n, k = sp["shape"]
            arr[i] = LinearTask(self._x(sp, x, x14).data_ptr(), out.data_ptr(), k, n, int(sp["block_start"]), 0)
        need = int(self.lib.voom_nf12_linear_batch_scratch_bytes(ctypes.byref(arr), len(self.specs), self.M))
        return arr, need

    def step_device(self, stream_ptr: int):
        """All seven projections in one voom_nf12_linear_batch launch."""
        import ctypes

        from voom_b200._lib import check

        if getattr(self, "_batch", None) is None or self._batch[0] is not self.outs:
            arr, need = self._tasks(self.x, self.x14, self.outs)
            scr = self.torch.empty(max(need, 1), dtype=self.torch.uint8, device=self.dev)
            self._batch = (self.outs, arr, need, scr)
        _, arr, need, scr = self._batch
        check(self.lib.voom_nf12_linear_batch(ctypes.byref(arr), len(self.specs), self.M, self.enc.data_ptr(),
                                              int(self.entry["file_bytes"]), int(self.entry["header_bytes"]),
                                              scr.data_ptr(), need, self.status.data_ptr(), stream_ptr),
              "voom_nf12_linear_batch")

    def verify(self) -> bool:
        torch = self.torch
        if int(self.status.item()):
            return False
        dense = self.nf12.decode_layer(self.enc, self.entry)
        for sp, out in zip(self.specs, self.outs):
            w = dense[sp["name"]].float()
            ref = self._x(sp, self.x, self.x14).float() @ w.T
            if float((out.float() - ref).norm() / ref.norm()) > 1e-2:
                return False
        return True

    def extra(self, stream, steps: int, flush) -> dict:
        """Whole-layer decode to BF16 (one voom_nf12_decode launch) and the fused
        linear at 8 activation rows."""
        torch = self.torch
        lib = self.lib
        out = torch.empty(int(self.entry["output_value_count"]), dtype=torch.int16, device=self.dev)
        st = torch.zeros(1, dtype=torch.int32, device=self.dev)

        def dec():
            lib.voom_nf12_decode(self.enc.data_ptr(), int(self.entry["file_bytes"]), int(self.entry["header_bytes"]),
                                 0, int(self.entry["block_count"]), 0, out.data_ptr(), out.numel(), st.data_ptr(),
                                 int(stream.cuda_stream))

        def timed(fn):
            fn()
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for a, b in ev:
                flush.fill_(5)
                a.record(stream)
                fn()
                b.record(stream)
            torch.cuda.synchronize()
            return sum(a.elapsed_time(b) for a, b in ev) / steps

        ms = timed(dec)
        ok = int(st.item()) == 0
        res = {"layer_decode": {"value": round(self.raw_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s decoded",
                                "ms_per_step": round(ms, 5), "hbm_gbs": round((len(self.payload) + self.raw_bytes)
                                                                              / (ms * 1e-3) / 1e9, 1),
                                "status_ok": ok}}
        if self.M != 8:
            w8 = C5Nf12.__new__(C5Nf12)
            w8.__dict__.update(self.__dict__)
            w8.M = 8
            g = torch.Generator().manual_seed(99)
            w8.x = torch.randn((8, 4096), generator=g).to(torch.bfloat16).to(self.dev)
            w8.x14 = torch.randn((8, 14336), generator=g).to(torch.bfloat16).to(self.dev)
            w8.outs = [torch.empty((8, sp["shape"][0]), dtype=torch.bfloat16, device=self.dev) for sp in self.specs]
            w8._batch = None
            ms8 = timed(lambda: w8.step_device(int(stream.cuda_stream)))
            res["fused_linear_M8"] = {"value": round(self.raw_bytes / (ms8 * 1e-3) / 1e9, 2), "unit": self.unit,
                                      "ms_per_step": round(ms8, 5), "correct": w8.verify()}
        return res

    def step_e2e(self):
        """Public API: activations from pinned host memory, the layer's seven
        projections through nf12.linear_batch (one launch), outputs back to
        pinned host memory."""
        x = self.x_host.to(self.dev, non_blocking=True)
        x14 = self.x14_host.to(self.dev, non_blocking=True)
        outs = self.nf12.linear_batch([(self._x(sp, x, x14), sp) for sp in self.specs], self.enc, self.entry,
                                      status=self.status)
        for o, oh in zip(outs, self.out_host):
            oh.copy_(o, non_blocking=True)
        return 2 * self.M * (4096 + 14336), sum(2 * self.M * sp["shape"][0] for sp in self.specs)

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """Oracle (numpy restatement of the block decode) of the q projection
        plus an fp32 matmul, one projection per thread, until `budget_s`."""
        from concurrent.futures import ThreadPoolExecutor

        from oracle import nf12 as onf

        sp = self.specs[0]
        n, k = sp["shape"]
        x = self.x.float().cpu().numpy()
        hb = int(self.entry["header_bytes"])

        def one(_):
            bits = onf.decode_span(self.payload, hb, int(sp["block_start"]), int(sp["block_count"]),
                                   int(sp["output_offset"]), n * k)
            return x @ onf.bf16_bits_to_f32(bits).reshape(n, k).T

        done = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while time.perf_counter() - t0 < budget_s:
                list(pool.map(one, range(threads)))
                done += threads
        dt = time.perf_counter() - t0
        return {"value": done * n * k * 2 / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{done} q_proj ({n}x{k}) oracle decodes + fp32 matmuls of {self.M} row(s) on {threads} "
                          f"thread(s), {dt:.1f} s"}

    def config(self) -> dict:
        return {"workload": self.name, "matrices": [[n, k] for _, n, k in self.SHAPES], "tokens": self.M,
                "encoded_bytes": len(self.payload), "bf16_bytes": self.raw_bytes,
                "ratio": round(self.raw_bytes / len(self.payload), 4),
                "l2": "flushed between steps (512 MiB write); the 327 MB stream exceeds L2"}


class C6KvPaged:
    """Config 5: the PagedKVCache spill/reload codec.  `pages` KV pages of 16
    positions x 8 KV heads x 128 head_dim BF16 (K and V N(0, 1) x a per-page,
    per-head scale U(0.5, 4)), spilled in the reference's compressed format
    (`.kvz`: pickle of {"shape", "k": zstd level 1 of K, "v": zstd level 1 of
    V}, runtime/kv_paged.py:77-91) on host threads.  A step reloads every
    page: all 2 x `pages` frames in one batched GPU decode.  Metric: decoded
    KV bytes per second."""

    metric = "BF16 weight-page decode GB/s (bit-exact)"
    unit = "GB/s"
    dtype = "u8"
    data = ("synthetic (seeded torch, generated on the device): K and V BF16 N(0, 1) x per-page per-head "
            "U(0.5, 4)")

    def __init__(self, device, rank: int, pages: int = 65536):
        import torch

        from voom_b200.formats import zstd_gpu
        from voom_b200.runtime import kv_paged

        self.torch = torch
        self.dev = device
        self.kv = kv_paged
        self.n_pages = pages
        self.name = f"c6_kv_paged_{pages}"
        H, P, D = 8, 16, 128
        g = torch.Generator(device=device).manual_seed(2026 + 7919 * rank)
        self.raw = torch.empty((pages, 2, 1, H, P, D), dtype=torch.bfloat16, device=device)
        chunk = 4096
        for a in range(0, pages, chunk):
            n = min(chunk, pages - a)
            x = torch.randn((n, 2, 1, H, P, D), generator=g, device=device)
            s = torch.rand((n, 2, 1, H, 1, 1), generator=g, device=device) * 3.5 + 0.5
            self.raw[a:a + n] = (x * s).to(torch.bfloat16)
        host = self.raw.view(torch.int16).cpu().numpy().view(np.uint16)
        self.spill_threads = os.cpu_count() or 8
        t0 = time.perf_counter()
        self.blobs = kv_paged.spill_pages_compressed(host[:, 0], host[:, 1], threads=self.spill_threads)
        self.spill_s = time.perf_counter() - t0
        del host
        self.page_bytes = 2 * H * P * D
        frames = []
        for b in self.blobs:
            d = pickle.loads(b)
            frames += [d["k"], d["v"]]
        jobs = np.zeros(len(frames), dtype=zstd_gpu.JOB_DTYPE)
        src = 0
        for i, f in enumerate(frames):
            jobs[i] = (src, len(f), i * self.page_bytes, self.page_bytes, 0, 0, 0)
            src += len(f)
        self.comp = np.frombuffer(b"".join(frames), np.uint8)
        self.plan = zstd_gpu.ZstdPlan(self.comp, jobs)
        self.batch = zstd_gpu.ZstdBatch(self.plan, device)
        self.src = _dev_upload(self.comp, device)
        self.out = torch.empty(len(frames) * self.page_bytes, dtype=torch.uint8, device=device)
        self.raw_bytes = self.out.numel()
        self.units_per_step = self.raw_bytes
        self.algo_bytes = self.comp.size + self.raw_bytes
        self.n_blocks = int(self.plan.info.n_blocks)
        self.n_seq = int(self.plan.info.n_seq)
        self.launches_per_step = 14  # direct literals, K0 K1 K1b K2 K3 K5 5xK4 patch K6

    def step_device(self, stream_ptr: int):
        self.batch.run(self.src, self.out, self.torch.cuda.current_stream(self.dev))

    def verify(self) -> bool:
        if self.batch.job_status().any():
            return False
        return bool(self.torch.equal(self.out, self.raw.view(-1).view(self.torch.uint8)))

    def extra(self, stream, steps: int, flush) -> dict:
        """The spill leg of the same pages.  GPU: every K and V frame made by
        the GPU encoder in one launch (device time of the encode kernel, CUDA
        events), and end to end through kv_paged.spill_pages_gpu (encode,
        device pack, one copy to the host, one pickle per page).  The frames
        are checked: the reference's load path (unpickle + libzstd) and the GPU
        reload both give the pages back.  Host: libzstd level 1 on a thread
        pool (the reference's own codec call), timed once at set-up."""
        torch = self.torch
        from oracle import vpack as ov
        from voom_b200.formats import zstd_gpu

        flat = self.raw.view(torch.uint8).reshape(-1)
        n = 2 * self.n_pages
        offs = np.arange(n, dtype=np.int64) * self.page_bytes
        lens = np.full(n, self.page_bytes, np.int64)
        plan = zstd_gpu.EncodePlan(offs, lens, self.dev)
        pinned = torch.empty(self.raw_bytes + 65536, dtype=torch.uint8).pin_memory()
        blobs = self.kv.spill_pages_gpu(self.raw[:, 0], self.raw[:, 1], pinned=pinned)
        bits = self.raw.view(torch.int16)
        ok = True
        for i in range(0, self.n_pages, max(1, self.n_pages // 64)):
            k, v = ov.kv_load(blobs[i])
            ref = bits[i].cpu().numpy().view(np.uint16)
            ok = ok and np.array_equal(k, ref[0]) and np.array_equal(v, ref[1])
        K, V = self.kv.reload_blobs(blobs, self.dev)
        ok = ok and bool(torch.equal(K.view(torch.int16), bits[:, 0]) and torch.equal(V.view(torch.int16), bits[:, 1]))
        comp = sum(len(b) for b in blobs)
        del K, V
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            flush.fill_(5)
            a.record(stream)
            plan.run(flat, stream)
            b.record(stream)
        torch.cuda.synchronize()
        enc_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        t0 = time.perf_counter()
        reps = max(1, min(3, steps))
        for _ in range(reps):
            self.kv.spill_pages_gpu(self.raw[:, 0], self.raw[:, 1], pinned=pinned)
        e2e_s = (time.perf_counter() - t0) / reps
        return {"spill_gpu": {"value": round(self.raw_bytes / (enc_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                              "ms_per_step": round(enc_ms, 4), "frames": n, "bit_exact_reload": ok,
                              "kvz_bytes": comp, "ratio_with_pickles": round(self.raw_bytes / comp, 4),
                              "e2e": {"value": round(self.raw_bytes / e2e_s / 1e9, 3), "unit": "GB/s",
                                      "seconds": round(e2e_s, 4),
                                      "how": "kv_paged.spill_pages_gpu: GPU encode, device pack, one copy to "
                                             "pinned host memory, a pickle per page"},
                              "how": "voom_zstd_encode over every K and V frame: Huffman-coded literal blocks "
                                     "(valid frames, not libzstd's bytes)"},
                "spill_host_libzstd": {"value": round(self.raw_bytes / self.spill_s / 1e9, 3), "unit": "GB/s",
                                       "seconds": round(self.spill_s, 3), "threads": self.spill_threads,
                                       "how": "kv_paged.spill_pages_compressed: zstd level 1 of K and V + pickle "
                                              "per page on host threads (the reference's codec call)"}}

    def step_e2e(self):
        """Public API: kv_paged.reload_blobs over the host-resident .kvz pages
        (parse, plan, one upload, one batched decode, status read back)."""
        self.kv.reload_blobs(self.blobs, self.dev)
        return int(self.comp.size), 4 * 2 * self.n_pages

    def cpu_sample(self, threads: int, budget_s: float) -> dict:
        """The reference reload (`_Page.load`: unpickle + zstd.decompress of K
        and V, kv_paged.py:98-113), pages spread over `threads` host threads,
        until `budget_s` of wall time."""
        from concurrent.futures import ThreadPoolExecutor

        from oracle import vpack as ov

        k, v = ov.kv_load(self.blobs[0])
        ref = self.raw[0].view(self.torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(k, ref[0]) and np.array_equal(v, ref[1])
        step = 1024
        done, i = 0, 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as pool:
            while time.perf_counter() - t0 < budget_s:
                sl = [self.blobs[(i + j) % self.n_pages] for j in range(step)]
                i += step
                for kk, _ in pool.map(ov.kv_load, sl):
                    done += 2 * kk.nbytes
        dt = time.perf_counter() - t0
        return {"value": done / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{done // self.page_bytes // 2} page reloads (.kvz unpickle + libzstd decompress of K "
                          f"and V) on {threads} thread(s), {dt:.1f} s"}

    def config(self) -> dict:
        return {"workload": self.name, "pages": self.n_pages, "page_shape": [1, 8, 16, 128], "tensors_per_page": 2,
                "frames": 2 * self.n_pages, "zstd_blocks": self.n_blocks, "sequences": self.n_seq,
                "compressed_bytes": int(self.comp.size), "raw_bytes": int(self.raw_bytes),
                "ratio": round(self.raw_bytes / self.comp.size, 4), "zstd_level": 1,
                "l2": "flushed between steps (512 MiB write); inputs and output exceed L2"}


def _dev_upload(arr, device):
    from voom_b200 import _device

    return _device.upload(arr, device)


WORKLOADS = {"c1_rans": C1Rans, "c2_vpack": C2Vpack, "c3_moe": C3Moe, "c4_moe_ep": C4MoeEP, "c5_nf12": C5Nf12,
             "c6_kv_paged": C6KvPaged}
DEFAULT_WORKLOAD = "c2_vpack"


# ------------------------------------------------------------------- main
ZSTD_KERNELS = {1: "zstd_direct_literals", 2: "zstd_block_decode", 3: "zstd_seq_scan", 4: "zstd_job_scan",
                5: "zstd_block_execute", 6: "zstd_output", 7: "zstd_resolve (all passes)", 8: "zstd_patch",
                9: "zstd_checksum", 10: "zstd_block_literals"}


def zstd_kernel_times(w, steps: int, flush, stream) -> dict | None:
    """Mean ms per step of every zstd kernel (CUDA events recorded by the
    library after each launch, voom_zstd_set_timing), outside the timed loop."""
    import ctypes

    import torch
    from voom_b200._lib import load

    if not hasattr(w, "batch"):
        return None
    lib = load()
    lib.voom_zstd_set_timing(1)
    ms = np.zeros(512, np.float32)
    ids = np.zeros(512, np.uint32)
    tot: dict = {}
    for i in range(steps):
        flush.fill_(i & 0xFF)
        w.step_device(int(stream.cuda_stream))
        n = lib.voom_zstd_kernel_times(ms.ctypes.data_as(ctypes.c_void_p), ids.ctypes.data_as(ctypes.c_void_p), 512)
        for k in range(max(n, 0)):
            name = ZSTD_KERNELS.get(int(ids[k]), str(int(ids[k])))
            tot[name] = tot.get(name, 0.0) + float(ms[k])
    torch.cuda.synchronize()
    lib.voom_zstd_set_timing(0)
    return {k: round(v / steps, 4) for k, v in tot.items()}


def dist_init():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _ref_archive(layers: int):
    """Config 2's vpack bodies built with numpy and libzstd only (through the
    oracle), so the reference arm maps none of this repository's libraries:
    the same tensors (seeded by name), the reference's body layout (hi plane
    zstd level 1, then the raw lo plane, formats/packed.py:125-358)."""
    import zlib

    from oracle import vpack as ov

    h, i, hd, vocab = 576, 1536, 64, 49152
    q, kv = 9 * hd, 3 * hd
    specs = [("model.embed_tokens.weight", (vocab, h))]
    for layer in range(layers):
        p = f"model.layers.{layer}."
        specs += [(p + "input_layernorm.weight", (h,)), (p + "self_attn.q_proj.weight", (q, h)),
                  (p + "self_attn.k_proj.weight", (kv, h)), (p + "self_attn.v_proj.weight", (kv, h)),
                  (p + "self_attn.o_proj.weight", (h, q)), (p + "post_attention_layernorm.weight", (h,)),
                  (p + "mlp.gate_proj.weight", (i, h)), (p + "mlp.up_proj.weight", (i, h)),
                  (p + "mlp.down_proj.weight", (h, i))]
    specs.append(("model.norm.weight", (h,)))

    def make(spec):
        name, shape = spec
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.02)
        u = x.view(np.uint32)
        bits = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
        a = bits.reshape(-1).view(np.uint8)
        hi_z = ov.zstd_compress(a[1::2].tobytes(), 1)
        return {"dtype": "BF16", "shape": list(shape), "hi_z": len(hi_z), "lo": a.size // 2}, hi_z + a[0::2].tobytes(), bits

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        return list(pool.map(make, specs))


def _ref_decoder():
    """The reference's own formats.packed2.decode_body when a reference checkout
    is present (its compression.zstd import served by the ctypes shim over
    libzstd kept with the test fixtures), else the oracle's restatement."""
    sys.path.insert(0, str(ROOT))
    from tests.reference_checkout import reference_root

    root = reference_root()
    if root is not None:
        shim = str(ROOT / "tests" / "golden" / "_shim")
        for pth in (shim, str(root)):
            if pth not in sys.path:
                sys.path.insert(0, pth)
        import importlib

        mod = importlib.import_module("formats.packed2")
        return mod.decode_body, "reference", "formats/packed2.py decode_body of the reference checkout"
    from oracle import vpack as ov

    return ov.decode_body, "port", "oracle/vpack.py decode_body (restatement of formats/packed2.py:178-191)"


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU decode of config 2 on all host
    threads, rank 0 only (other ranks exit without work).  A step is one pass
    over the whole archive, bodies spread over the threads."""
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor

    threads = os.cpu_count() or 1
    items = _ref_archive(args.c2_layers)
    decode, kind, what = _ref_decoder()
    raw_bytes = sum(b.nbytes for _, _, b in items)
    arch_bytes = sum(len(body) for _, body, _ in items)
    for (head, body, bits) in items[:3]:  # the decoder reproduces the tensors
        assert np.array_equal(np.asarray(decode(head, body), np.uint8).reshape(-1), bits.reshape(-1).view(np.uint8))
    times = []
    with ThreadPoolExecutor(max_workers=threads) as pool:
        order = sorted(range(len(items)), key=lambda k: -len(items[k][1]))
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            n = sum(pool.map(lambda k: np.asarray(decode(items[k][0], items[k][1])).size, order))
            dt = time.perf_counter() - t0
            assert n == raw_bytes
            if step >= args.warmup:
                times.append(dt)
    ms = statistics.median(times) * 1e3
    v = raw_bytes / (ms * 1e-3) / 1e9
    sample = (f"{args.steps} passes over the {len(items)}-body config-2 archive ({raw_bytes} B decoded per pass) "
              f"with {what} on {threads} host threads")
    line = {
        "metric": C2Vpack.metric, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": C2Vpack.data,
        "config": {"workload": C2Vpack.name, "tensors": len(items), "archive_bytes": int(arch_bytes),
                   "raw_bytes": int(raw_bytes), "ratio": round(raw_bytes / arch_bytes, 4), "zstd_level": 1},
        "impl": "reference",
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure(w, args, stream, flush, world: int, clocks: bool = True) -> dict:
    """Bit-exactness check, warm-up, `args.steps` timed device steps (CUDA
    events on the launching stream, L2 flushed between steps), then the same
    number of end-to-end steps through the public API.  Every rank takes the
    same collective steps; times are the max over ranks."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device())
    sptr = int(stream.cuda_stream)
    w.step_device(sptr)
    torch.cuda.synchronize()
    ok = w.verify()
    if world > 1:
        t = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = bool(t.item())
    if not ok:
        raise SystemExit(f"bench: {type(w).__name__} device result is not exact")
    for _ in range(args.warmup):
        flush.fill_(1)
        w.step_device(sptr)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device()) if clocks else None
    if sampler:
        sampler.start()
    marks = []
    if hasattr(w, "_mark"):
        del w._mark
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    coll = []
    for i in range(args.steps):
        flush.fill_(i & 0xFF)  # evict the previous step's data from L2
        starts[i].record(stream)
        w.step_device(sptr)
        ends[i].record(stream)
        if hasattr(w, "_mark"):
            marks.append(w._mark)
        if hasattr(w, "collective_ms"):
            coll.append(getattr(w, "_ev", []))
    torch.cuda.synchronize()
    clock_rec = sampler.stop() if sampler else None
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    ms = sum(step_ms) / len(step_ms)
    part_ms = sum(a.elapsed_time(m) for a, m in zip(starts, marks)) / len(marks) if marks else None
    coll_ms = sum(a.elapsed_time(b) for ev in coll for a, b in ev) / len(coll) if any(coll) else None
    vals = [ms, part_ms or 0.0, coll_ms or 0.0]
    coll = coll if coll_ms is not None else []
    if world > 1:
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
    out = {"ms": vals[0], "step_ms": step_ms, "part_ms": vals[1] if marks else None,
           "coll_ms": vals[2] if coll else None, "clocks": clock_rec}
    # end to end through the public API, pinned host buffers, copies inside
    for _ in range(2):
        w.step_e2e()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    bi = bo = 0
    for _ in range(args.steps):
        bi, bo = w.step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    out.update(e2e_ms=e2e_ms, h2d=bi, d2h=bo)
    return out


def sum_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v)], device=torch.device("cuda", torch.cuda.current_device()), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def roofline(achieved: float, peaks: dict, peaks_kind: str, algo: int, workload: str, note: str) -> dict:
    prof = profiled_traffic(workload)
    return {"bound": "hbm", "achieved": round(achieved, 3), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 5), "traffic": prof[0] if prof else None,
            "traffic_unit": "DRAM bytes per step (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "traffic_source": prof[1] if prof else None, "algorithmic_bytes_per_step": int(algo),
            "achieved_note": note, "peak_kind": f"{peaks_kind} (hbm_gbs)"}


def moe_record(w, r: dict, world: int, peaks, peaks_kind, cpu: dict | None, extra: dict) -> dict:
    """Nested record of one MoE workload (tok/s, roofline, e2e, NCCL share)."""
    ms = r["ms"]
    algo = sum_over_ranks(w.algo_bytes, world)
    rec = {"value": round(w.units_per_step / (ms * 1e-3), 3), "unit": "tok/s", "ms_per_step": round(ms, 5),
           "roofline": roofline(algo / world / (ms * 1e-3) / 1e9, peaks, peaks_kind, int(algo / world),
                                extra.get("workload", ""),
                                "compressed pages of the routed experts on a GPU + activations in and out, per step"
                                ", mean over ranks / step time"),
           "e2e": {"value": round(w.units_per_step / (r["e2e_ms"] * 1e-3), 3), "unit": "tok/s",
                   "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
           "cpu_baseline": cpu, "clocks": r["clocks"],
           "gpu_launches": getattr(w, "launches_per_step", 1) * 1}
    if r.get("coll_ms") is not None:
        rec["collective"] = {"op": "NCCL reduce-scatter of the token-major route rows + all-gather of the combined "
                                   "rows (waits for the slowest rank included)", "ms_per_step": round(r["coll_ms"], 5),
                             "share_of_step": round(r["coll_ms"] / ms, 4)}
    rec.update(extra)
    return rec


def headline(args, world, rank, local, dev):
    """The default run: config 2 decode GB/s as the line's value, with nested
    records for config 4 (expert parallel, T = 1, 8, 64) and, on one GPU,
    config 3 (T = 1, 8)."""
    import torch
    import torch.distributed as dist

    peaks, peaks_kind = load_peaks()
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    host_threads = os.cpu_count() or 1

    w = C2Vpack(dev, rank, layers=args.c2_layers, world=world)
    r = measure(w, args, stream, flush, world)
    ms = r["ms"]
    value = w.units_per_step / (ms * 1e-3) / 1e9
    e2e_value = w.units_per_step / (r["e2e_ms"] * 1e-3) / 1e9
    dec_ms = r["part_ms"]
    algo = sum_over_ranks(w.algo_bytes, world)
    achieved = algo / world / (dec_ms * 1e-3) / 1e9
    kernel_ms = zstd_kernel_times(w, args.steps, flush, stream) if args.kernel_times else None
    cpu = w.cpu_sample(host_threads, budget_s=args.cpu_seconds) if (rank == 0 and world == 1) else None
    line = {
        "metric": w.metric, "value": round(value, 4), "unit": w.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": w.scaling, "vs_baseline": None, "dtype": w.dtype,
        "data": w.data, "config": w.config(),
        "roofline": roofline(achieved, peaks, peaks_kind, int(algo / world), w.config()["workload"],
                             "per GPU: compressed + decoded bytes of its share / its decode time (the "
                             "all-gather excluded)"),
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 4), "unit": w.unit, "h2d_bytes_per_step": r["h2d"],
                "d2h_bytes_per_step": r["d2h"]},
        "gpu_launches": args.steps * w.launches_per_step, "clocks": r["clocks"],
        "step_ms_min": round(min(r["step_ms"]), 5), "step_ms_max": round(max(r["step_ms"]), 5),
        "decode_ms_per_step": round(dec_ms, 5),
        **({"kernel_ms": kernel_ms} if kernel_ms is not None else {}),
    }
    if world == 1 and not args.no_cpu:
        line["repack"] = w.repack_leg(host_threads)
    if world > 1:
        line["collective"] = {"op": "NCCL all-gather of the decoded bodies", "bytes_per_rank": int(w.gather_bytes),
                              "ms_per_step": round(ms - dec_ms, 5), "share_of_step": round(1 - dec_ms / ms, 4)}
    del w
    torch.cuda.empty_cache()

    if not args.no_moe:
        c4 = C4MoeEP(dev, rank, world=world, tokens=tuple(args.c4_tokens), layers=args.c4_layers)
        recs = {}
        for T in args.c4_tokens:
            st = c4.for_tokens(T)
            rr = measure(st, args, stream, flush, world)
            cpu4 = None
            if rank == 0 and world == 1 and T in (1, 8):
                cpu4 = st.cpu_sample(host_threads, budget_s=args.cpu_seconds / 2)
                cpu4["cpu_model"] = cpu_model()
            recs[f"T{T}"] = moe_record(st, rr, world, peaks, peaks_kind, cpu4, {
                "tokens": T, "workload": f"c4_moe_ep_T{T}",
                "local_routed_experts_per_step": st.local_routed,
                "distinct_experts_per_layer": st.distinct_per_layer})
        line["moe_ep"] = {"metric": c4.metric, "config": c4.config(), "scaling": "strong", "by_tokens": recs}
        del c4
        torch.cuda.empty_cache()
        if world == 1:
            store = None
            c3 = {}
            for T in (1, 8):
                w3 = C3Moe(dev, 0, tokens=T, store=store)
                store = w3.store
                rr = measure(w3, args, stream, flush, world)
                cpu3 = w3.cpu_sample(host_threads, budget_s=args.cpu_seconds / 2)
                cpu3["cpu_model"] = cpu_model()
                c3[f"T{T}"] = moe_record(w3, rr, 1, peaks, peaks_kind, cpu3,
                                         {"tokens": T, "workload": w3.name,
                                          "distinct_experts_per_step": getattr(w3, "distinct", None)})
            line["c3_moe"] = {"metric": C3Moe.metric, "config": w3.config(), "by_tokens": c3}
            del w3, store
            torch.cuda.empty_cache()
            w5 = C6KvPaged(dev, 0, pages=args.kv_pages)
            r5 = measure(w5, args, stream, flush, 1)
            ms5 = r5["ms"]
            cpu5 = w5.cpu_sample(host_threads, budget_s=args.cpu_seconds / 2)
            cpu5["cpu_model"] = cpu_model()
            line["kv_paged"] = {
                "metric": "KV page reload GB/s (decoded K/V bytes, bit-exact)", "value": round(
                    w5.units_per_step / (ms5 * 1e-3) / 1e9, 3), "unit": "GB/s", "ms_per_step": round(ms5, 5),
                "config": w5.config(),
                "roofline": roofline(w5.algo_bytes / (ms5 * 1e-3) / 1e9, peaks, peaks_kind, int(w5.algo_bytes),
                                     w5.config()["workload"], "compressed + decoded bytes / step time"),
                "e2e": {"value": round(w5.units_per_step / (r5["e2e_ms"] * 1e-3) / 1e9, 3), "unit": "GB/s",
                        "h2d_bytes_per_step": r5["h2d"], "d2h_bytes_per_step": r5["d2h"]},
                "cpu_baseline": cpu5, "clocks": r5["clocks"], **w5.extra(stream, args.steps, flush)}
    if rank == 0:
        print(json.dumps(line), flush=True)


def single(args, world, rank, local, dev):
    """--workload X: one workload's line (profiling and development runs)."""
    import torch

    peaks, peaks_kind = load_peaks()
    wl = WORKLOADS[args.workload]
    if wl is C3Moe:
        w = wl(dev, rank, tokens=args.tokens)
    elif wl is C5Nf12:
        w = wl(dev, rank, tokens=args.tokens)
    elif wl is C4MoeEP:
        w = wl(dev, rank, world=world, tokens=(args.tokens,), layers=args.c4_layers).for_tokens(args.tokens)
    elif wl is C2Vpack:
        w = wl(dev, rank, layers=args.c2_layers, world=world)
    elif wl is C6KvPaged:
        w = wl(dev, rank, pages=args.kv_pages)
    else:
        w = wl(dev, rank)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    if args.device_only:
        sptr = int(stream.cuda_stream)
        w.step_device(sptr)
        torch.cuda.synchronize()
        if not w.verify():
            raise SystemExit("bench: device result is not exact")
        for _ in range(args.warmup):
            w.step_device(sptr)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in ev:
            flush.fill_(2)
            a.record(stream)
            w.step_device(sptr)
            b.record(stream)
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
        kernel_ms = zstd_kernel_times(w, args.steps, flush, stream) if args.kernel_times else None
        if rank == 0:
            name = w.config()["workload"] if hasattr(w, "config") else type(w).__name__
            line = {"device_only": True, "workload": name, "steps": args.steps, "ms_per_step": round(ms, 5)}
            if kernel_ms is not None:
                line["kernel_ms"] = kernel_ms
            print(json.dumps(line), flush=True)
        return
    r = measure(w, args, stream, flush, world)
    ms = r["ms"]
    mult = 1 if getattr(w, "replicated_units", False) else world
    if w.unit == "GB/s":
        value = w.units_per_step * mult / (ms * 1e-3) / 1e9
        e2e_value = w.units_per_step * mult / (r["e2e_ms"] * 1e-3) / 1e9
    else:
        value = w.units_per_step * mult / (ms * 1e-3)
        e2e_value = w.units_per_step * mult / (r["e2e_ms"] * 1e-3)
    extra = w.extra(stream, args.steps, flush) if hasattr(w, "extra") else {}
    algo = sum_over_ranks(w.algo_bytes, world)
    t_ms = r["part_ms"] or ms
    cfg = w.config() if hasattr(w, "config") else w.c4.config()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = w.cpu_sample(os.cpu_count() or 1, budget_s=args.cpu_seconds)
    if rank == 0:
        line = {
            "metric": getattr(w, "metric", getattr(getattr(w, "c4", None), "metric", "")), "value": round(value, 4),
            "unit": w.unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": getattr(w, "scaling", "weak"),
            "vs_baseline": None, "dtype": getattr(w, "dtype", "bf16"), "data": getattr(w, "data", ""),
            "config": cfg,
            "roofline": roofline(algo / world / (t_ms * 1e-3) / 1e9, peaks, peaks_kind, int(algo / world),
                                 cfg["workload"], "algorithmic bytes per GPU / step time"),
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 4), "unit": w.unit, "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"]},
            "gpu_launches": args.steps * getattr(w, "launches_per_step", 1), "clocks": r["clocks"],
            **({"collective_ms_per_step": round(r["coll_ms"], 5)} if r.get("coll_ms") is not None else {}),
            **extra,
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="one workload only (default: config 2 as the line's value with nested config-4 and "
                         "config-3 records)")
    ap.add_argument("--ref-seconds", type=float, default=4.0)
    ap.add_argument("--cpu-seconds", type=float, default=6.0)
    ap.add_argument("--tokens", type=int, default=1, help="--workload c3_moe / c4_moe_ep / c5_nf12: tokens")
    ap.add_argument("--c2-layers", type=int, default=30, help="c2_vpack: layers of the archive (30 = config 2)")
    ap.add_argument("--c4-tokens", type=int, nargs="+", default=[1, 8, 64], help="config-4 token counts")
    ap.add_argument("--c4-layers", type=int, default=4, help="config-4 routers per step")
    ap.add_argument("--kv-pages", type=int, default=65536, help="c6_kv_paged: KV pages (65536 = config 5)")
    ap.add_argument("--no-moe", action="store_true", help="default run: config 2 only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs and the repack leg")
    ap.add_argument("--kernel-times", action="store_true",
                    help="zstd workloads: after the timed steps, time `--steps` more steps with a CUDA event after "
                         "every kernel launch and report the mean ms per kernel per step ('kernel_ms')")
    ap.add_argument("--device-only", action="store_true",
                    help="--workload runs: parity check, warm-up and timed device steps only (the run the ncu "
                         "captures in profiles/ use); prints a short line")
    args = ap.parse_args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    import torch
    import torch.distributed as dist

    world, rank, local = dist_init()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    try:
        if args.workload is None:
            headline(args, world, rank, local, dev)
        else:
            single(args, world, rank, local, dev)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
