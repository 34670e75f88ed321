"""Benchmark of the B200 binary-UNet forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the Bi-Real dual-skip binary UNet (base width 32, 120 bands, 3
classes, random weights from seed 0 with the benchmark's distributions) on
4096 independent 32x32x120 float32 patches per GPU (seeded synthetic
inputs, bnn_synth.h). A step is one forward over the GPU's 4096 patches.
Under torchrun each rank takes its own slice of patch indices
[rank*4096, (rank+1)*4096) (weak scaling, no collective on the data path);
timing is the max over ranks.

  value : patches/s with the inputs already in HBM (device-pointer API),
          CUDA events on the launching stream around the K timed steps
  e2e   : patches/s through the public host-pointer API bnn_forward_batch,
          pinned host input -> logits in pinned host memory, every step
  roofline : the dominant kernel family (the 17 fused binary convs, int8
          tensor cores) from per-kernel CUDA events over the same timed
          steps, against the int8 dense tensor peak (2x the measured bf16
          rate); rooflines.* also give the first conv and the host link
  cpu_baseline : the reference engine compiled from its own sources
          (oracle/_ref/ref_bench), all host cores, bounded sample

--impl reference times only the reference CPU engine (rank 0).

--workload scene runs BASELINE config 3 instead: 16 scene cubes of
956x684x120 float32 (seeded synthetic values, cube index as the patch key)
through the patched forward (non-overlapping zero-padded 32x32 tiles,
30x22 = 660 per cube), the cubes split over the ranks (strong scaling of the
fixed 16-cube job); value = tiles/s with the cubes in HBM, e2e = tiles/s
through bnn_forward_patched from host memory (2 cubes per rank).

--workload react runs BASELINE config 4: the v3 ReAct real-highway UNet
(base 16) on 1024 patches of 64x64x120 per GPU, against the reference's
ReAct engine (oracle/_ref/ref_bench_react) as the CPU arm.

--workload stem runs config 2's batch through the v2 spectral-stem variant
of the network (16-channel 1x1 stem + real fold, enc1.conv1 binary), against
the reference's stem engine (oracle/_ref/ref_bench_stem) as the CPU arm.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "UNet patches/s (32x32x120)"
STEM_C = 16                 # v2 stem width: the reference's default (python/bnn2c spectral stem)
REACT_C = 16                # v3 ReAct base width: the reference's default (python/bnn2c/blob_react.py C0_DEFAULT)
REACT_METRIC = "ReAct UNet patches/s (64x64x120)"
FFMA_PER_CLK_SM = 128       # fp32 fused multiply-adds / clock / SM (nominal; probe: 119)
SEED_MODEL, SEED_INPUT = 0, 1
POPC_PER_CLK_SM = 16        # 32-bit population count results / clock / SM (CUDA guide; probe: 15.6)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the 17 binary-conv
# launches of one forward of the default workload at 512 patches, from one ncu
# capture of that forward's 20 launches (the kernels with the register-weight head
# and the e2m1 rule of 2 / 8 words); scaled by patches in the bench line
BCONV_DRAM_BYTES_PER_512 = 23.7e6
# the same for the first conv's main kernel (its 251.66 MB input read once)
REALIN_DRAM_BYTES_PER_512 = 256.1e6
# bit planes the 17 binary convs read and write per 32x32 patch at base 32
# (inputs, concat halves, outputs and pooled outputs)
BCONV_ALGO_BYTES_PER_PATCH = 58112
MMA_SYNC_I8_PER_CLK_SM = 1951  # int8 MACs / clock / SM of mma.sync m16n8k32 (measured by a probe kernel)


def read_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.out = tempfile.TemporaryFile(mode="w+")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_info():
    model = "unknown"
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return model, os.cpu_count() or 1


REF_BUILD = {"march": None}  # which reference build ran (set by run_ref)


def run_ref(name, argv, threads):
    """Run a reference timing driver built from the reference sources: the
    -march=native build (the reference Makefile's flags, csrc/Makefile:9-11)
    when it runs on this host, else the portable -march=x86-64-v3 one. Returns
    (CompletedProcess, None) or (None, reason)."""
    last = None
    for sub, march in (("native", "native"), ("", "x86-64-v3")):
        exe = os.path.join(ROOT, "oracle", "_ref", sub, name)
        if not os.path.exists(exe):
            continue
        r = subprocess.run([exe] + [str(a) for a in argv], capture_output=True, text=True,
                           env=dict(os.environ, OMP_NUM_THREADS=str(threads)))
        if r.returncode < 0:  # killed by a signal: an instruction this host lacks
            last = f"{name} ({march}) died with signal {-r.returncode}"
            continue
        if r.returncode != 0:
            return None, f"{name} failed: {r.stderr.strip()[-200:]}"
        REF_BUILD["march"] = march
        return r, None
    return None, last or f"oracle/_ref/{name} not built (needs the reference tree at build time)"


def ref_bench(blob_path, n, H, W, procs, steps, warm, first=0, stem=False, name=None):
    """Reference engine (compiled from the reference sources) on the host:
    the v1 engine, with stem=True the v2 spectral-stem engine, or the driver
    `name` (ref_bench_react: the v3 ReAct engine)."""
    name = name or ("ref_bench_stem" if stem else "ref_bench")
    r, err = run_ref(name, [blob_path, n, H, W, procs, SEED_INPUT, steps, warm, first], 1)
    if r is None:
        return None, err
    secs = [float(ln.split()[2]) for ln in r.stdout.splitlines() if ln.startswith("step ")]
    return secs, None


# ---------------------------------------------------------------- config 1
SWEEP_C = (64, 128, 256, 512)
SWEEP_H = (128, 64, 32, 16)
SWEEP_N = 64
SEED_SWEEP = 11


def sweep_layer(C, seed, pool):
    """Random weights (uniform bits, kidx-packed as in the blob) and folds
    (rule P >= t, t uniform in [-2C, 2C]) of one sweep layer."""
    import numpy as np

    rng = np.random.default_rng(seed)
    nw = (9 * C + 63) // 64
    packed = np.frombuffer(rng.bytes(C * nw * 8), np.uint64).reshape(C, nw).copy()
    if (9 * C) % 64:
        packed[:, -1] &= np.uint64((1 << ((9 * C) % 64)) - 1)

    def fold():
        return {"type": np.ones(C, np.int32), "t": rng.integers(-2 * C, 2 * C + 1, C).astype(np.int32),
                "lo": np.zeros(C, np.int32), "hi": np.zeros(C, np.int32)}

    return packed, fold(), (fold() if pool else None)


def ref_sweep_point(C, H, pool, budget):
    """Seconds per image of the reference's own layer (bconv_dispatch +
    apply_fold_int [+ maxpool_P + apply_fold_int]), all host cores."""
    _, cores = cpu_info()
    r, err = run_ref("ref_bench_bconv", [C, H, int(pool), budget], cores)
    if r is None:
        return None, err
    kv = dict(ln.split(None, 1) for ln in r.stdout.splitlines() if " " in ln)
    return float(kv["image_s"]), int(kv["images"])


def run_sweep(local, reps=10, warm=3, ref_budget=0.3, cpu=True):
    """the isolated fused binary conv layer (3x3, pad 1,
    stride 1, Cin = Cout = C) over C in {64,128,256,512} x H = W in
    {128,64,32,16}, batch 64, without and with the 2x2 max-pool of P, through
    bnn_bconv_layer_run on device buffers. Each timed run is one launch,
    bracketed by CUDA events on its stream, after an L2 flush (a 256 MB
    write); the median of `reps` runs is reported. 1 bitop = 1 binary MAC =
    Cout*H*W*Cin*9 per image (the reference profiler's work unit)."""
    import numpy as np
    import torch

    import bnns_to_c_b200 as bn

    peaks = read_peaks()
    bf16 = peaks.get("bf16_tflops")
    i8 = bf16 * 1e3 if bf16 else 2.25e6          # G int8 MAC/s: 2x the bf16 MAC rate
    hbm = peaks.get("hbm_gbs") or 6650.0
    props = torch.cuda.get_device_properties(local)
    popc = props.multi_processor_count * POPC_PER_CLK_SM * 32 * (peaks.get("sm_max_mhz") or 1965.0) * 1e6 / 1e9
    stream = torch.cuda.Stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    model, cores = cpu_info()
    shapes, tot_mac, tot_ms, tot_ref = [], 0.0, 0.0, 0.0
    for C in SWEEP_C:
        for pool in (False, True):
            packed, f1, f2 = sweep_layer(C, SEED_SWEEP + C + int(pool), pool)
            L = bn.BconvLayer(local, C, C, packed, f1, f2)
            for H in SWEEP_H:
                N, W, cw = SWEEP_N, H, C // 32
                din = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, H, W, cw), dtype=torch.int32, device="cuda")
                dout = torch.empty((N, H, W, cw), dtype=torch.int32, device="cuda")
                dpool = torch.empty((N, H // 2, W // 2, cw), dtype=torch.int32, device="cuda") if pool else None
                torch.cuda.synchronize()
                with torch.cuda.stream(stream):
                    for _ in range(warm):
                        L.run(din, N, H, W, dout, dpool, stream=stream)
                    kern = bn.bconv_last_kernel()
                    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                          for _ in range(reps)]
                    for r in range(reps):
                        flush.fill_(r & 0xFF)
                        ev[r][0].record(stream)
                        L.run(din, N, H, W, dout, dpool, stream=stream)
                        ev[r][1].record(stream)
                stream.synchronize()
                ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
                mac = float(N) * H * W * C * C * 9
                nbytes = N * H * W * C // 8 * 2 + (N * (H // 2) * (W // 2) * C // 8 if pool else 0) + C * C * 9 // 8
                g = mac / (ms * 1e6)
                row = {"C": C, "H": H, "pool": pool, "ms": round(ms, 5), "gbitops": round(g, 1),
                       "frac_int8": round(g / i8, 4), "frac_e2m1": round(g / (2 * i8), 4),
                       "frac_popc": round(g / popc, 3), "hbm_gbs": round(nbytes / (ms * 1e6), 1),
                       "kernel": kern}
                if cpu:
                    per, err = ref_sweep_point(C, H, pool, ref_budget)
                    if per is not None:
                        row["ref_ms_per_batch"] = round(per * N * 1e3, 3)
                        row["ref_gbitops"] = round(mac / (per * N) / 1e9, 2)
                        row["speedup"] = round(per * N * 1e3 / ms, 1)
                        tot_ref += per * N * 1e3
                    else:
                        row["ref_error"] = err
                shapes.append(row)
                tot_mac += mac
                tot_ms += ms
                del din, dout, dpool
            L.close()
    del flush
    g_all = tot_mac / (tot_ms * 1e6)
    out = {
        "metric": "binary-conv Gbitop/s (config 1 sweep, 1 bitop = 1 binary MAC)",
        "gbitops": round(g_all, 1), "ms_total": round(tot_ms, 3),
        "frac_int8": round(g_all / i8, 4), "frac_e2m1": round(g_all / (2 * i8), 4),
        "peak_int8_gmacs": round(i8, 1), "peak_source": "int8 dense tensor rate = 2x the measured cuBLAS bf16 rate "
        "(MEASURED_PEAKS.json)" if bf16 else "fallback", "popc_peak_gbitops": round(popc, 1),
        "config": {"C": list(SWEEP_C), "H=W": list(SWEEP_H), "batch": SWEEP_N, "pool": [False, True],
                   "thresholds": "P >= t, t ~ U[-2C, 2C]", "timing": f"median of {reps} single launches, "
                   "CUDA events, L2 flushed (256 MB write) before each", "data": "uniform random bits"},
        "shapes": shapes,
    }
    if cpu and tot_ref:
        out["reference"] = {"ms_total": round(tot_ref, 1), "gbitops": round(tot_mac / (tot_ref * 1e6), 2),
                            "speedup": round(tot_ref / tot_ms, 1), "cores": cores, "march": REF_BUILD["march"],
                            "sample": f"images of each shape timed for up to {ref_budget} s after one untimed image "
                                      f"(at most 64), scaled to the batch of {SWEEP_N}; OpenMP on {cores} threads, "
                                      f"{model}"}
    return out


# ---------------------------------------------------------------- config 0
def cli_forward_ms(exe, blob_path, out_path, reps, threads):
    """Median forward ms that a csrc/main.c-style CLI reports for one 32x32
    'rand' patch (srand(1234) uniform [-1, 1] input, `reps` timed forwards)."""
    r = subprocess.run([exe, blob_path, "rand", out_path, "32", "32", str(reps)], capture_output=True, text=True,
                       env=dict(os.environ, OMP_NUM_THREADS=str(threads)))
    if r.returncode != 0:
        return None, f"{os.path.basename(exe)} rc {r.returncode}: {r.stderr.strip()[-160:]}"
    for ln in r.stderr.splitlines():
        if ln.startswith("# forward"):
            return float(ln.split(":", 1)[1].split()[0]), None
    return None, "no forward line"


def run_single(m, local, reps=50, ref_reps=5, cpu=True):
    """one 32x32x120 patch, batch 1 (latency).
    cli: this engine's bnn_infer (csrc/main.c semantics: bnn_forward on host
    buffers, median of `reps`), the call an existing caller of main.c makes;
    device: bnn_forward_device with N = 1 from HBM (graph replay, CUDA events);
    reference: its own CLI built from its sources, 1 thread and all cores."""
    import numpy as np
    import torch

    import bnns_to_c_b200 as bn

    out = {"metric": "single-patch forward latency (32x32x120, batch 1)", "unit": "us/patch"}
    with tempfile.TemporaryDirectory() as td:
        blob = os.path.join(td, "m.blob")
        with open(blob, "wb") as f:
            f.write(model_blob())
        mine, err = cli_forward_ms(bn.CLI_PATH, blob, os.path.join(td, "ours.bin"), reps, 1)
        out["cli_us"] = round(mine * 1e3, 1) if mine is not None else None
        if err:
            out["cli_error"] = err
        # the same call in-process (ctypes), pageable host buffers
        x = np.random.default_rng(3).standard_normal((120, 32, 32)).astype(np.float32)
        y = np.empty((3, 32, 32), np.float32)
        L = bn.lib()
        for _ in range(5):
            L.bnn_forward(m.handle, x.ctypes.data, 32, 32, y.ctypes.data)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            L.bnn_forward(m.handle, x.ctypes.data, 32, 32, y.ctypes.data)
            ts.append(time.perf_counter() - t0)
        out["bnn_forward_us"] = round(statistics.median(ts) * 1e6, 1)
        din = torch.from_numpy(x[None]).cuda()
        dout = torch.empty((1, 3, 32, 32), dtype=torch.float32, device="cuda")
        st = torch.cuda.Stream()
        for _ in range(5):
            m.forward_device(local, din, 1, 32, 32, dout, st)
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            m.forward_device(local, din, 1, 32, 32, dout, st)
        e1.record(st)
        st.synchronize()
        out["device_us"] = round(e0.elapsed_time(e1) * 1e3 / reps, 1)
        if cpu:
            _, cores = cpu_info()
            ref = {}
            for th in (1, cores):
                r, err = run_ref("bnn_infer", [blob, "rand", os.path.join(td, "ref.bin"), 32, 32, ref_reps], th)
                ms = None
                if r is not None:
                    for ln in r.stderr.splitlines():
                        if ln.startswith("# forward"):
                            ms = float(ln.split(":", 1)[1].split()[0])
                ref[f"threads_{th}_us"] = round(ms * 1e3, 1) if ms is not None else err
            ref["march"] = REF_BUILD["march"]
            out["reference"] = ref
            if mine is not None and os.path.exists(os.path.join(td, "ref.bin")):
                a = np.fromfile(os.path.join(td, "ours.bin"), np.float32)
                b = np.fromfile(os.path.join(td, "ref.bin"), np.float32)
                out["cli_logits_identical"] = bool(a.shape == b.shape and np.array_equal(a.view(np.uint32),
                                                                                         b.view(np.uint32)))
            if mine is not None and isinstance(ref.get("threads_1_us"), float):
                out["speedup_vs_reference_1_thread"] = round(ref["threads_1_us"] / out["cli_us"], 1)
    return out


def model_blob(stem=0):
    from bnns_to_c_b200 import blob as B

    return B.blob_bytes(B.random_model(32, 120, 3, seed=SEED_MODEL, rules="baseline", stem_channels=stem))


def react_blob():
    from bnns_to_c_b200 import blob_react as BR

    return BR.react_blob_bytes(BR.random_react_model(REACT_C, 120, 3, seed=SEED_MODEL))


def variant(args):
    """(stem channels, metric, workload name) of the network benched."""
    shape = f"{args.patches}x{args.H}x{args.W}x120"
    if args.workload == "stem":
        return STEM_C, "v2 spectral-stem UNet patches/s (32x32x120)", f"stem{STEM_C}_unet_c32_{shape}"
    return 0, METRIC, f"unet_c32_{shape}"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.workload == "react":
        return run_reference_react(args)
    stem, metric, wname = variant(args)
    data = model_blob(stem)
    with tempfile.NamedTemporaryFile(suffix=".blob", delete=False) as f:
        f.write(data)
        path = f.name
    model, cores = cpu_info()
    n = cores * args.ref_per_core
    secs, err = ref_bench(path, n, args.H, args.W, cores, args.steps, max(0, min(args.warmup, 1)), stem=bool(stem))
    os.unlink(path)
    if secs is None:
        print(json.dumps({"impl": "reference", "unavailable": err}))
        return 0
    v = n * len(secs) / sum(secs)
    sample = (f"{n} patches per step ({args.ref_per_core} per core), {cores} single-threaded processes, "
              f"-O3 -march={REF_BUILD['march']}, {model}")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(v, 3), "unit": "patches/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * sum(secs) / len(secs), 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "b1+f32", "data": "synthetic",
        "config": {"workload": wname, "base_channels": 32, "H": args.H, "W": args.W,
                   "bands": 120, "classes": 3, "patches_per_step": n},
        "cpu_baseline": {"value": round(v, 3), "unit": "patches/s", "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "patches/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


def gpu_affinity(local):
    """Pin this process to the host CPUs local to its GPU (the PCI device's
    local_cpulist), before any pinned host buffer is touched, so the staging
    pages and copy threads sit on the GPU's NUMA node. Returns what was done."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(local)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{bus}"
        cpus = set()
        for part in open(f"{base}/local_cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        node = open(f"{base}/numa_node").read().strip()
        if cpus and cpus != set(os.sched_getaffinity(0)):
            os.sched_setaffinity(0, cpus)
            return {"pci": bus, "numa_node": node, "cpus": len(cpus), "pinned": True}
        return {"pci": bus, "numa_node": node, "cpus": len(cpus), "pinned": False}
    except Exception as e:  # no sysfs entry (containers), keep the default
        return {"error": str(e)[:120]}


def run_ours(args):
    import numpy as np
    import torch

    import bnns_to_c_b200 as bn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    def maxall(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    P, H, W = args.patches, args.H, args.W
    stem, metric, wname = variant(args)
    affinity = gpu_affinity(local)
    bn.set_bconv_kernel(args.bconv)
    bn.set_first_conv_kernel(args.first)
    m = (bn.StemModel if stem else bn.Model)(data=model_blob(stem))
    m.set_devices([local])
    first = rank * P
    din = torch.empty((P, 120, H, W), dtype=torch.float32, device="cuda")
    dout = torch.empty((P, 3, H, W), dtype=torch.float32, device="cuda")
    bn.synth_device(local, SEED_INPUT, first, P, 120, H, W, din)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    # ---------------- device-resident value: CUDA-graph replays, no profiler ----------------
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            m.forward_device(local, din, P, H, W, dout, stream)
        e1.record(stream)
        stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    dev_ms = maxall(e0.elapsed_time(e1))
    clocks = clk.summary()
    # the same K-step region repeated (run-to-run spread of the headline; not the headline itself)
    reps_ms = []
    for _ in range(args.repeats):
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            m.forward_device(local, din, P, H, W, dout, stream)
        f1.record(stream)
        stream.synchronize()
        reps_ms.append(maxall(f0.elapsed_time(f1)))
    # ---------------- per-kernel CUDA events: separate profiled steps (eager launches) ----------------
    m.profile(True)
    m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    m.profile_reset()
    for _ in range(args.prof_steps):
        m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    recs = m.profile_records()
    m.profile(False)

    # ---------------- end to end through the public host API ----------------
    e2e_s, same, h2d_gbs, h2d_agg_gbs = None, None, None, None
    if not args.no_e2e:
        hin = torch.empty((P, 120, H, W), dtype=torch.float32, pin_memory=True)
        hin.copy_(din.cpu())
        hout = torch.empty((P, 3, H, W), dtype=torch.float32, pin_memory=True)
        hin_np, hout_np = hin.numpy(), hout.numpy()
        for _ in range(max(1, args.warmup)):
            m.forward_batch(hin_np, out=hout_np)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            m.forward_batch(hin_np, out=hout_np)
        e2e_s = maxall(time.perf_counter() - t0)
        barrier()
        # the two paths agree (same patches, same logits)
        same = bool(torch.equal(hout.view(torch.int32), dout.cpu().view(torch.int32)))
        # the host link by itself: one pinned 2 GB host->device copy, CUDA events
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        din.copy_(hin, non_blocking=True)
        torch.cuda.synchronize()
        c0.record()
        din.copy_(hin, non_blocking=True)
        c1.record()
        torch.cuda.synchronize()
        h2d_gbs = hin.numel() * 4 / (c0.elapsed_time(c1) * 1e6)
        # the box's aggregate host->device ceiling: every rank copies its 2 GB at
        # the same moment (after a barrier); time = the slowest rank's copy
        barrier()
        c0.record()
        din.copy_(hin, non_blocking=True)
        c1.record()
        torch.cuda.synchronize()
        agg_s = maxall(c0.elapsed_time(c1) / 1e3)
        h2d_agg_gbs = world * hin.numel() * 4 / agg_s / 1e9

    if rank == 0:
        peaks = read_peaks()
        props = torch.cuda.get_device_properties(local)
        sms = props.multi_processor_count
        max_mhz = clocks.get("sm_max_mhz") or peaks.get("sm_max_mhz") or 1965.0
        by_op = {}
        for r in recs:
            o = by_op.setdefault(r["op"], {"ms": 0.0, "work": 0.0, "calls": 0})
            o["ms"] += r["ms"]; o["work"] += r["work"]; o["calls"] += r["calls"]
        total_ms = sum(o["ms"] for o in by_op.values())
        clk = max_mhz * 1e6
        popc_peak = sms * POPC_PER_CLK_SM * 32 * clk / 1e9              # G bitMAC/s
        mma_sync_peak = sms * MMA_SYNC_I8_PER_CLK_SM * clk / 1e9         # G int8 MAC/s, legacy path
        bf16 = peaks.get("bf16_tflops")
        tensor_i8_peak = bf16 * 1e3 if bf16 else 2.25e6                  # G int8 MAC/s = 2x bf16 MAC rate
        b = by_op.get("bconv", {"ms": 1e-9, "work": 0})
        r_ = by_op.get("conv_real", {"ms": 1e-9, "work": 0})
        bconv_ach = b["work"] / (b["ms"] * 1e6)   # work = Cout*H*W*Cin*9 binary MACs (reference PROF unit)
        # first conv: int8 MACs the tensor cores execute (3 planes x 128 padded bands)
        real_macs = 3 * 128 / 120 * r_["work"]
        real_ach = real_macs / (r_["ms"] * 1e6)
        launches_per_fwd = m.launches(P, H, W)
        chunks = -(-P // 256)
        value = P * world * args.steps / (dev_ms / 1e3)
        e2e = P * world * args.steps / e2e_s if e2e_s else None
        model, cores = cpu_info()
        cpu = None
        # the reference on the host cores: rank 0 of a single-GPU run only
        if world == 1 and not args.no_cpu_baseline:
            with tempfile.NamedTemporaryFile(suffix=".blob", delete=False) as f:
                f.write(model_blob(stem))
                path = f.name
            n = cores * args.ref_per_core
            secs, err = ref_bench(path, n, H, W, cores, 1, 0, stem=bool(stem))
            os.unlink(path)
            if secs:
                cpu = {"value": round(n / secs[0], 3), "unit": "patches/s", "cores": cores, "kind": "reference",
                       "sample": f"{n} patches of the same workload, {cores} single-threaded processes of the "
                                 f"reference engine built from its sources (-O3 -march={REF_BUILD['march']}), "
                                 f"{model}"}
            else:
                cpu = {"value": None, "unit": "patches/s", "cores": cores, "kind": "reference", "sample": err}
        frac_split = {k: round(v["ms"] / total_ms, 4) for k, v in by_op.items()} if total_ms else {}
        line = {
            "metric": metric, "value": round(value, 1), "unit": "patches/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "b1+f32",
            "data": "synthetic",
            "config": {"workload": wname, "base_channels": 32, "bands": 120, "classes": 3,
                       "H": H, "W": W, "patches_per_gpu": P, "global_batch": P * world,
                       "parallelism": f"patch-shard x{world}",
                       "l2": f"inputs > L2 ({P * 120 * H * W * 4 / 1e9:.2f} GB read per step)"},
            "e2e": {"value": round(e2e, 1) if e2e else None, "unit": "patches/s",
                    "h2d_bytes_per_step": P * 120 * H * W * 4,
                    "d2h_bytes_per_step": P * 3 * H * W * 4, "api": "bnn_forward_batch (pinned host buffers)",
                    "matches_device_path": same,
                    "h2d_link_gbs": round(h2d_gbs, 2) if h2d_gbs else None,
                    # per GPU: this rank's share of the e2e rate against its own link
                    "frac_of_h2d_link": round(e2e / world * 120 * H * W * 4 / (h2d_gbs * 1e9), 4)
                    if (e2e and h2d_gbs) else None,
                    "h2d_aggregate_gbs": round(h2d_agg_gbs, 2) if h2d_agg_gbs else None,
                    "frac_of_h2d_aggregate": round(e2e * 120 * H * W * 4 / (h2d_agg_gbs * 1e9), 4)
                    if (e2e and h2d_agg_gbs) else None,
                    "h2d_aggregate_how": "all ranks copy their pinned 2 GB input at once after a barrier; "
                                         "world x bytes / the slowest rank's copy time",
                    "affinity": affinity,
                    # this repo's kernels in the end-to-end timed region (the batch runs in
                    # 256-patch chunks, one graph replay each)
                    "gpu_launches": None if args.no_e2e else launches_per_fwd * args.steps * chunks},
            # this repo's kernels launched in the device-resident timed region (per rank)
            "gpu_launches": launches_per_fwd * args.steps,
            "device_wait_timeouts": bn.device_wait_timeouts(local),
            "roofline": (
                {"bound": "tensor",
                 "kernel": ("bconv_ws_kernel + bconv_ws_pool_kernel (17 fused binary convs, tcgen05 int8, "
                            "persistent warp-specialised)") if args.bconv in ("tc", "tc8", "tc4", "tcx") else
                           "bconv_mma_kernel (17 fused binary convs, int8 mma.sync)",
                 "achieved": round(bconv_ach, 1), "peak": round(tensor_i8_peak, 1),
                 "unit": "Gbitop/s (1 bitop = 1 binary MAC, run as one int8 MAC)",
                 "frac": round(bconv_ach / tensor_i8_peak, 4),
                 "traffic": round(BCONV_DRAM_BYTES_PER_512 * P / 512) if (H, W) == (32, 32) and not stem else None,
                 "traffic_scope": "DRAM bytes of the 17 binary-conv launches of one forward (ncu, 512-patch "
                                  "capture scaled by patches); their bit planes stay mostly in L2",
                 "algorithmic_bytes": BCONV_ALGO_BYTES_PER_PATCH * P if (H, W) == (32, 32) and not stem else None,
                 "peak_source": "int8 dense tensor rate = 2x the measured cuBLAS bf16 rate in MEASURED_PEAKS.json"
                 if bf16 else "fallback 2.25 P int8 MAC/s",
                 "frac_of_mma_sync_measured": round(bconv_ach / mma_sync_peak, 4),
                 "frac_of_popc_peak": round(bconv_ach / popc_peak, 4),
                 # the e2m1 layers (default: the deeper 64/128/256-channel ones) have twice the int8 rate
                 "frac_of_e2m1_peak": round(bconv_ach / (2 * tensor_i8_peak), 4),
                 # what bounds them, from ncu (not this run): the tensor-core operand interface
                 "tc_interface_busy_ncu": {"dec1.conv1 bconv_ws_kernel<32,8,0,4>, 4096 patches": 0.785,
                                           "source": "ncu --set full, one launch of the 4096-patch forward"},
                 "time_share": frac_split.get("bconv")}
                if args.bconv in ("tc", "tc8", "tc4", "tcx", "mma") else
                {"bound": "popc", "kernel": "bconv3x3_kernel (17 fused binary convs, XOR + POPC)",
                 "achieved": round(bconv_ach, 1), "peak": round(popc_peak, 1), "unit": "Gbitop/s",
                 "frac": round(bconv_ach / popc_peak, 4), "traffic": None,
                 "peak_source": f"nominal {sms} SMs x {POPC_PER_CLK_SM} POPC/clk x 32 bit x {max_mhz:.0f} MHz "
                                "(probe: 15.6 POPC/clk/SM)",
                 "time_share": frac_split.get("bconv")}),
            "rooflines": {
                "conv_real": {"bound": "hbm", "kernel": "stem_fold_kernel (v2 stem 1x1 + real fold, exact fp32 order)",
                              "achieved": round(P * 120 * H * W * 4 * args.prof_steps / (r_["ms"] * 1e6), 1),
                              "peak": peaks.get("hbm_gbs"), "unit": "GB/s (input bands read once)",
                              "frac": round(P * 120 * H * W * 4 * args.prof_steps / (r_["ms"] * 1e6)
                                            / peaks["hbm_gbs"], 4) if peaks.get("hbm_gbs") else None,
                              "time_share": frac_split.get("conv_real")} if stem else
                {"bound": "tensor",
                              "kernel": {"tc": "realin_ws_kernel (tcgen05, nine shifted taps)",
                                         "tcn": "realin_dxn_kernel (tcgen05, column taps in N)",
                                         "tx": "realin_tx_kernel (tcgen05, weights in M, positions in N)",
                                         "mma": "realin_mma_kernel (mma.sync)"}[args.first]
                              + " + realin_fixup_kernel",
                              "achieved": round(real_ach, 1), "peak": round(tensor_i8_peak, 1),
                              "unit": "G int8 MAC/s executed (3 planes x 128 bands x 9 taps x 32 ch per pixel)",
                              "frac": round(real_ach / tensor_i8_peak, 4),
                              "frac_of_mma_sync_measured": round(real_ach / mma_sync_peak, 4),
                              # the same kernels as an input-read (HBM) roofline
                              "hbm_gbs": round(P * 120 * H * W * 4 * args.prof_steps / (r_["ms"] * 1e6), 1),
                              "frac_of_hbm": round(P * 120 * H * W * 4 * args.prof_steps / (r_["ms"] * 1e6)
                                                   / peaks["hbm_gbs"], 4) if peaks.get("hbm_gbs") else None,
                              "traffic": round(REALIN_DRAM_BYTES_PER_512 * P / 512)
                              if (H, W) == (32, 32) and not stem else None,
                              # what bounds it, from ncu (not this run): the tensor-core operand interface
                              "tc_interface_busy_ncu": {"realin_ws_kernel<32,7>, 512 patches": 0.719,
                                                        "source": "ncu --set full, one launch at 512 patches"}
                              if args.first == "tc" else None,
                              "time_share": frac_split.get("conv_real")},
                "hbm_input": {"bytes_per_step": P * 120 * H * W * 4, "peak_gbs": peaks.get("hbm_gbs"),
                              "min_ms": round(P * 120 * H * W * 4 / (peaks.get("hbm_gbs", 6538.9) * 1e6), 4)},
            },
            "per_kernel_ms": {r["label"]: round(r["ms"] / r["calls"], 4) for r in recs},
            "per_layer_frac": {r["label"]: round(r["work"] / (r["ms"] * 1e6) / tensor_i8_peak, 4)
                               for r in recs if r["op"] == "bconv"},
            "per_kernel_source": "CUDA events around each launch in separate eager (non-graph) steps after "
                                 "the timed region; their sum runs ~3% above the graph-replayed step, so the "
                                 "per-kernel fractions are slightly pessimistic",
            "repeats_ms_per_step": [round(t / args.steps, 4) for t in reps_ms],
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if world == 1 and not args.no_single:
            line["single"] = run_single(m, local, cpu=not args.no_cpu_baseline)
        if world == 1 and not args.no_sweep:
            line["sweep"] = run_sweep(local, cpu=not args.no_cpu_baseline)
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()
    return 0


def run_sweep_line(args):
    """--workload sweep: BASELINE config 1 alone, as its own JSON line
    (rank 0 of a one-GPU run)."""
    import torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    import bnns_to_c_b200 as bn

    bn.set_bconv_kernel(args.bconv)
    with ClockSampler(local) as clk:
        sw = run_sweep(local, reps=max(3, args.steps), warm=args.warmup, cpu=not args.no_cpu_baseline)
    line = {"metric": sw["metric"], "value": sw["gbitops"], "unit": "Gbitop/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sw["ms_total"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "b1", "data": "synthetic",
            "config": dict(sw["config"], workload="bconv_sweep_C64-512_H16-128_b64"),
            "roofline": {"bound": "tensor", "achieved": sw["gbitops"], "peak": sw["peak_int8_gmacs"],
                         "unit": "Gbitop/s (1 binary MAC run as one int8 or e2m1 MAC)", "frac": sw["frac_int8"],
                         "frac_of_e2m1_peak": sw["frac_e2m1"], "traffic": None},
            "cpu_baseline": ({"value": sw["reference"]["gbitops"], "unit": "Gbitop/s",
                              "cores": sw["reference"]["cores"], "kind": "reference",
                              "sample": sw["reference"]["sample"]} if "reference" in sw else None),
            "clocks": clk.summary(), "sweep": sw}
    print(json.dumps(line))
    return 0


def run_scene(args):
    import torch

    import bnns_to_c_b200 as bn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def maxall(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    H, W, Pt, total = 956, 684, 32, args.cubes
    mine = list(range(rank, total, world))  # this rank's cubes
    tiles = -(-H // Pt) * -(-W // Pt)
    m = bn.Model(data=model_blob())
    m.set_devices([local])
    cubes = [torch.empty((120, H, W), dtype=torch.float32, device="cuda") for _ in mine]
    logs = [torch.empty((3, H, W), dtype=torch.float32, device="cuda") for _ in mine]
    for c, i in zip(cubes, mine):
        bn.synth_device(local, SEED_INPUT, 1000 + i, 1, 120, H, W, c)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            for c, lg in zip(cubes, logs):
                m.forward_patched_device(local, c, H, W, lg, Pt, stream)
    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            for c, lg in zip(cubes, logs):
                m.forward_patched_device(local, c, H, W, lg, Pt, stream)
        e1.record(stream)
        stream.synchronize()
    if dist:
        dist.barrier()
    dev_ms = maxall(e0.elapsed_time(e1))
    # end to end from host memory (a bounded sample: up to 2 cubes per rank)
    ns = min(2, len(mine))
    hc = [torch.empty((120, H, W), dtype=torch.float32, pin_memory=True) for _ in range(ns)]
    hl = [torch.empty((3, H, W), dtype=torch.float32, pin_memory=True) for _ in range(ns)]
    for i in range(ns):
        hc[i].copy_(cubes[i].cpu())
    for i in range(ns):
        m.forward_patched(hc[i].numpy(), Pt, out=hl[i].numpy())
    same = all(bool(torch.equal(hl[i].view(torch.int32), logs[i].cpu().view(torch.int32))) for i in range(ns))
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for i in range(ns):
            m.forward_patched(hc[i].numpy(), Pt, out=hl[i].numpy())
    e2e_s = maxall(time.perf_counter() - t0)
    job_tiles = tiles * total
    if rank == 0:
        line = {
            "metric": "scene tiles/s (956x684x120 cubes, 32x32 tiles)",
            "value": round(job_tiles * args.steps / (dev_ms / 1e3), 1), "unit": "tiles/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "b1+f32",
            "data": "synthetic",
            "config": {"workload": "scene_16x956x684x120_tiles32", "cubes": total, "tiles_per_cube": tiles,
                       "cube_mb": round(120 * H * W * 4 / 1e6, 1), "parallelism": f"cube-shard x{world}",
                       "l2": "inputs > L2 (each cube 314 MB)"},
            "e2e": {"value": round(tiles * ns * world * args.steps / e2e_s, 1), "unit": "tiles/s",
                    "h2d_bytes_per_step": 120 * H * W * 4 * ns * world, "d2h_bytes_per_step": 3 * H * W * 4 * ns * world,
                    "api": "bnn_forward_patched (pinned host cubes)", "matches_device_path": same,
                    "sample": f"{ns} cubes per rank"},
            # per cube and step: the tile gather, the batched forward, the stitch
            # (a cube's tiles fit one forward chunk), rank 0's share
            "gpu_launches": len(mine) * args.steps * (2 + m.launches(tiles, Pt, Pt)),
            "clocks": clk.summary(),
        }
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()
    return 0


def run_reference_react(args):
    """Reference arm of BASELINE config 4: the reference's v3 ReAct engine
    (oracle/_ref/ref_bench_react) on the host cores, 64x64 patches."""
    H = W = 64
    with tempfile.NamedTemporaryFile(suffix=".blob", delete=False) as f:
        f.write(react_blob())
        path = f.name
    model, cores = cpu_info()
    n = cores * args.ref_per_core
    secs, err = ref_bench(path, n, H, W, cores, args.steps, max(0, min(args.warmup, 1)), name="ref_bench_react")
    os.unlink(path)
    if secs is None:
        print(json.dumps({"impl": "reference", "unavailable": err}))
        return 0
    v = n * len(secs) / sum(secs)
    print(json.dumps({
        "impl": "reference", "metric": REACT_METRIC, "value": round(v, 3), "unit": "patches/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * sum(secs) / len(secs), 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "b1+f32", "data": "synthetic",
        "config": {"workload": f"react_c{REACT_C}_64x64x120", "base_channels": REACT_C, "H": H, "W": W,
                   "bands": 120, "classes": 3, "patches_per_step": n},
        "cpu_baseline": {"value": round(v, 3), "unit": "patches/s", "cores": cores, "kind": "reference",
                         "sample": f"{n} patches per step, {cores} single-threaded processes, {model}"},
        "e2e": {"value": round(v, 3), "unit": "patches/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


def run_react(args):
    """the v3 ReAct UNet (base 16, random weights from
    seed 0 with the config's distributions) on 1024 patches of 64x64x120 per
    GPU per step."""
    import torch

    import bnns_to_c_b200 as bn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    def maxall(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    P, H, W = args.react_patches, 64, 64
    bn.set_bconv_kernel(args.bconv)
    m = bn.ReactModel(data=react_blob())
    din = torch.empty((P, 120, H, W), dtype=torch.float32, device="cuda")
    dout = torch.empty((P, 3, H, W), dtype=torch.float32, device="cuda")
    bn.synth_device(local, SEED_INPUT, rank * P, P, 120, H, W, din)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            m.forward_device(local, din, P, H, W, dout, stream)
        e1.record(stream)
        stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    dev_ms = maxall(e0.elapsed_time(e1))
    clocks = clk.summary()
    # per-kernel CUDA events: separate profiled steps (eager launches)
    m.profile(True)
    m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    m.profile_reset()
    for _ in range(args.prof_steps):
        m.forward_device(local, din, P, H, W, dout, stream)
    stream.synchronize()
    recs = m.profile_records()
    m.profile(False)
    e2e_s, same = None, None
    if not args.no_e2e:
        hin = torch.empty((P, 120, H, W), dtype=torch.float32, pin_memory=True)
        hin.copy_(din.cpu())
        hout = torch.empty((P, 3, H, W), dtype=torch.float32, pin_memory=True)
        for _ in range(max(1, args.warmup)):
            m.forward_batch(hin.numpy(), out=hout.numpy())
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            m.forward_batch(hin.numpy(), out=hout.numpy())
        e2e_s = maxall(time.perf_counter() - t0)
        same = bool(torch.equal(hout.view(torch.int32), dout.cpu().view(torch.int32)))
    if rank == 0:
        peaks = read_peaks()
        props = torch.cuda.get_device_properties(local)
        sms = props.multi_processor_count
        max_mhz = clocks.get("sm_max_mhz") or peaks.get("sm_max_mhz") or 1965.0
        by_op = {}
        for r in recs:
            o = by_op.setdefault(r["op"], {"ms": 0.0, "work": 0.0})
            o["ms"] += r["ms"]
            o["work"] += r["work"]
        total_ms = sum(o["ms"] for o in by_op.values()) or 1e-9
        fma_peak = sms * FFMA_PER_CLK_SM * max_mhz * 1e6 / 1e9          # G FMA/s
        bf16 = peaks.get("bf16_tflops")
        tensor_i8_peak = bf16 * 1e3 if bf16 else 2.25e6
        hbm = peaks.get("hbm_gbs") or 6538.9

        def rate(op):
            o = by_op.get(op, {"ms": 1e-9, "work": 0.0})
            return o["work"] / (o["ms"] * 1e6), o["ms"] / total_ms

        real_ach, real_share = rate("conv_real")
        proj_ach, proj_share = rate("proj")
        bconv_ach, bconv_share = rate("bconv")
        epi_ach, epi_share = rate("epi")
        value = P * world * args.steps / (dev_ms / 1e3)
        model, cores = cpu_info()
        cpu = None
        # the reference on the host cores: rank 0 of a single-GPU run only
        if world == 1 and not args.no_cpu_baseline:
            with tempfile.NamedTemporaryFile(suffix=".blob", delete=False) as f:
                f.write(react_blob())
                path = f.name
            n = cores * args.ref_per_core
            secs, err = ref_bench(path, n, H, W, cores, 1, 0, name="ref_bench_react")
            os.unlink(path)
            cpu = ({"value": round(n / secs[0], 3), "unit": "patches/s", "cores": cores, "kind": "reference",
                    "sample": f"{n} patches of the same workload, {cores} single-threaded processes of the "
                              f"reference ReAct engine built from its sources, {model}"} if secs else
                   {"value": None, "unit": "patches/s", "cores": cores, "kind": "reference", "sample": err})
        line = {
            "metric": REACT_METRIC, "value": round(value, 1), "unit": "patches/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "b1+f32",
            "data": "synthetic",
            "config": {"workload": f"react_c{REACT_C}_{P}x64x64x120", "base_channels": REACT_C, "bands": 120,
                       "classes": 3, "H": H, "W": W, "patches_per_gpu": P, "global_batch": P * world,
                       "parallelism": f"patch-shard x{world}",
                       "l2": f"inputs > L2 ({P * 120 * H * W * 4 / 1e9:.2f} GB read per step)"},
            "e2e": {"value": round(P * world * args.steps / e2e_s, 1) if e2e_s else None, "unit": "patches/s",
                    "h2d_bytes_per_step": P * 120 * H * W * 4, "d2h_bytes_per_step": P * 3 * H * W * 4,
                    "api": "bnn_forward_react_batch (pinned host buffers)", "matches_device_path": same},
            "gpu_launches": m.launches(P, H, W) * args.steps,
            "device_wait_timeouts": bn.device_wait_timeouts(local),
            "roofline": {"bound": "fp32", "kernel": "conv3_tma_kernel (enc1 real 3x3 conv, TMA-staged, exact fp32 order)",
                         "achieved": round(real_ach, 1), "peak": round(fma_peak, 1),
                         "unit": "G FMA/s (Cout x Cin x 9 per pixel)", "frac": round(real_ach / fma_peak, 4),
                         "traffic": None, "time_share": round(real_share, 4),
                         "peak_source": f"nominal {sms} SMs x {FFMA_PER_CLK_SM} FMA/clk x {max_mhz:.0f} MHz"},
            "rooflines": {
                "proj": {"bound": "fp32", "achieved": round(proj_ach, 1), "peak": round(fma_peak, 1),
                         "unit": "G FMA/s", "frac": round(proj_ach / fma_peak, 4), "time_share": round(proj_share, 4)},
                "bconv": {"bound": "tensor", "achieved": round(bconv_ach, 1), "peak": round(tensor_i8_peak, 1),
                          "unit": "Gbitop/s", "frac": round(bconv_ach / tensor_i8_peak, 4),
                          "time_share": round(bconv_share, 4)},
                "epi": {"bound": "hbm", "time_share": round(epi_share, 4), "peak_gbs": hbm},
                "hbm_input": {"bytes_per_step": P * 120 * H * W * 4,
                              "min_ms": round(P * 120 * H * W * 4 / (hbm * 1e6), 4)},
            },
            "per_kernel_ms": {r["label"]: round(r["ms"] / max(1, r["calls"]), 4) for r in recs},
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--patches", type=int, default=4096, help="patches per GPU per step")
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--W", type=int, default=32)
    ap.add_argument("--ref-per-core", type=int, default=4, help="reference sample: patches per host core")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-pointer leg (profiling runs)")
    ap.add_argument("--first", default="tc", choices=["tc", "mma", "tcn", "tx"],
                    help="first conv kernel: tcgen05 (default) or mma.sync")
    ap.add_argument("--bconv", default="tc", choices=["tc", "tc8", "tc4", "tcx", "popc", "mma"],
                    help="binary-conv kernels: tc = tcgen05 int8, e2m1 where measured faster (default), "
                         "tc8 = tcgen05 int8 throughout, tc4 = tcgen05 e2m1 for every non-pooled layer, "
                         "tcx = tc8 with the column taps in N at 32 channels, popc = XOR + POPC, "
                         "mma = mma.sync for every layer")
    ap.add_argument("--no-sweep", action="store_true", help="leave the config-1 binary-conv sweep out of the line")
    ap.add_argument("--no-single", action="store_true", help="leave the config-0 single-patch latency out")
    ap.add_argument("--repeats", type=int, default=4,
                    help="extra repeats of the K-step device region (spread only; the headline is the first)")
    ap.add_argument("--workload", default="unet", choices=["unet", "scene", "stem", "react", "sweep"],
                    help="unet: BASELINE config 2 (default); scene: config 3, whole cubes through the tiler; "
                         "stem: config 2's batch through the v2 spectral-stem variant (16-channel stem); "
                         "react: config 4, the v3 ReAct UNet on 64x64 patches")
    ap.add_argument("--react-patches", type=int, default=1024, help="react workload: patches per GPU per step")
    ap.add_argument("--prof-steps", type=int, default=2,
                    help="profiled steps after the timed region (per-kernel CUDA events, eager launches)")
    ap.add_argument("--cubes", type=int, default=16, help="scene workload: cubes in the job")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "scene":
        return run_scene(args)
    if args.workload == "react":
        return run_react(args)
    if args.workload == "sweep":
        return run_sweep_line(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
