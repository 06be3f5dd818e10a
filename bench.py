"""Benchmark of the sparse-pooling training step (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline metric's config): a Mode-A fp32
layer of N = 100,663,296 neurons, fan-in 8, D = 4096 inputs, G = 4096 mean-ReLU
pooling groups of 24,576 neurons, batch B = 1024; one step = forward + backward
(dX, dW, db) + fused Adam (beta = (0.9, 0.999), eps = 1e-8, lr = 1e-3, fp32
moments).  Inputs are synthetic: x ~ N(0,1), upstream gradient ~ N(0,1),
parameters from the layer's seeded init (seed 2 + rank, bias_std 0.1).

Multi-GPU (torchrun, one rank per GPU): rank r owns a contiguous slice of
groups; the pooled output is all-gathered and dX all-reduced over NCCL.  The
total work is fixed, so scaling is "strong"; ``value`` is the whole-job
throughput B*N / (max over ranks of the step time).

``value`` is device-timed (CUDA events, K steps, barrier + synchronize on both
sides) with inputs resident in HBM; parameters (5.2 GB) are far larger than
L2, so every pass streams them from HBM.  ``e2e`` is the same metric through
the public API with pinned host buffers (x and dy copied in, y copied out
every step).  ``roofline`` is for the dominant kernel (the backward), timed
with CUDA events on its launch stream.  ``cpu_baseline`` times the C oracle on
a bounded slice of the same workload on the host cores (rank 0, N = 1).

``--workload cover16`` times instead BASELINE config 4, the Cover-TopK/16 opt-in layer
(N = 50,331,648 neurons selected from a K64 envelope with w64 ~ N(0, 1/64) in BF16, D = 4096,
G = 2048 outputs, S = 64, R = 64, batch 512, seed 3): forward + backward through the layer on
1 GPU, with the forward and backward (dX-carrying) kernels timed separately.  fp32 parameters run
the tensor-core kernels on three-term bf16 splits by default (``--cover-kernels simt``: the fp32
SIMT kernels; ``t5`` / ``t5fwd`` / ``t5bwd``: the forward and / or backward on tcgen05 with TMEM
accumulators); ``--cover-dtype bf16`` stores bf16 parameters (the reference's arithmetic).

``--workload fwdbwd256`` times BASELINE config 2: the same 100M-neuron layer (seed 1, bias_std 0.1)
forward + backward at batch 256 through the layer API (no optimizer), forward and backward
kernels timed separately.

``--workload locality`` runs BASELINE config 5: a Mode-A layer with D = 16384, N = 100,663,296,
G = 8192 (seed 4), timed forward-only and forward + backward at batch 1, 32, 256, 1024 and 4096,
once with the reference's uniform index rule and once with windowed indices (each supergroup of
4096 consecutive neurons draws from its own random 512-wide input window; layout.windowed_indices).

``--workload modeb`` times Mode B (C neurons share one index record; the reference's
production mode and the configuration of its published RTX 3090 table): H = 100,000,000,
D = G = 1024, B = 8192, Mean(ReLU) and Max (identity, save_winners), fragment-packed storage,
fwd + bwd + fused Adam (fp32), for C = 8 and C = 64, plus Mean(ReLU) with
``PhysicalPlan(reduction="deterministic")`` (bitwise-repeatable backward) and
Mean(ReLU) with bf16 parameters and the optimizer's defaults (bf16 moments,
stochastic rounding), the precision of the published table.

``--impl reference`` times the reference's CPU path (the oracle port: the
reference's materialising PyTorch path does not fit 100M neurons) on the same
config, rank 0 only.

``--impl reference-gpu`` (comparator, not part of the driver contract) runs the unmodified
reference package placed in baseline/_ref on this GPU through its public API: with
``--workload modeb`` the published table's rows on its BF16 mma.sync CUDA kernels, with
``--workload sets`` its input-supergroup layers, with ``--workload cover16`` its Cover-TopK/16
layer on its BF16 K16 kernels, otherwise the headline Mode-A fp32 layer on its Triton kernels.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

D, N, G, B = 4096, 100_663_296, 4096, 1024
INDEX_RULE = "uniform"    # --index-rule: "uniform" (configs 2 / 3 as written) or "distinct" (the reference's init)
INDEX_RULES = {"distinct": "int16, distinct sorted per neuron (reference init rule)",
               "uniform": "int16 storage of the configs' uniform int32 rule: every index uniform in [0, D) with "
                          "replacement (D = 4096 fits int16)"}


@torch.no_grad()
def uniform_indices_(idx, seed):
    """Overwrite a Mode-A index tensor [G, NB, 8, 8] with BASELINE configs 2 / 3's rule as written: every index
    uniform in [0, D) with replacement, from a seeded generator on the tensor's device."""
    gen = torch.Generator(device=idx.device).manual_seed(seed)
    idx.copy_(torch.randint(0, D, idx.shape, generator=gen, device=idx.device).to(torch.int16))


def shard_layer(D_, N_, G_, dev, seed, bias_std=0.1, group=None):
    """The benchmarked GroupShardedLayer with the --index-rule's indices, in octet storage."""
    from granulelayer_b200.distributed import GroupShardedLayer

    if INDEX_RULE == "distinct":
        return GroupShardedLayer(D_, N_, G_, pooling="mean", device=dev, seed=seed, bias_std=bias_std, group=group)
    lay = GroupShardedLayer(D_, N_, G_, pooling="mean", device=dev, seed=seed, bias_std=bias_std, group=group,
                            neuron_order="slot")
    uniform_indices_(lay.indices, 1000 + seed + lay.rank)
    lay.order_kind = "octet"
    lay.reorder_neurons()
    return lay
K_FAN = 8
IDX_BYTES = 2
METRIC = "neuron-samples/s fwd+bwd+opt @100M fan-in-8, B=1024; % HBM roofline; 1/2/4/8 GPU"
UNIT = "neuron-samples/s"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per neuron per backward launch at B = 1024, from the ncu capture in
# BWD_PROFILE (512 x 24,576 neurons); the traffic grows with the neuron count, so a full launch is
# this figure times N.
BWD_PROFILE = "profiles/octet_kernels_g512.md"
BWD_DRAM_BYTES_PER_NEURON = (1.350285e9 + 0.532295e9) / (512 * 24576)   # the folded backward's capture


def param_bytes(n):
    return n * (K_FAN * 4 + K_FAN * IDX_BYTES + 4)


def gather_bytes(b, n):
    return b * n * K_FAN * 4


def peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def peak_bf16():
    """Dense bf16 tensor rate (TFLOP/s): the burst figure of MEASURED_PEAKS.json, else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def config_dict(world):
    return {"workload": "100M-neuron fan-in-8 Mode-A fp32 mean-ReLU layer: fwd+bwd+fused Adam step "
                        "(D=4096, N=100,663,296, G=4096 groups of 24,576, B=1024)",
            "D": D, "N": N, "G": G, "global_batch": B, "fan_in": K_FAN, "pool": "mean", "activation": "relu",
            "indices": INDEX_RULES[INDEX_RULE],
            "l2": "inputs larger than L2: 5.2 GB of parameters streamed from HBM every pass",
            "parallelism": f"group-shard x{world}" if world > 1 else "single GPU"}


class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML (read-only) in a thread, every 50 ms, so that even
    a sub-second timed region (8 GPUs: 10 steps of ~56 ms) yields about ten samples."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.index = index
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # noqa: BLE001
            self.error = f"{type(e).__name__}: {e}"
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.05)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)

    @staticmethod
    def max_clock_hz(index) -> float:
        """The GPU's maximum SM clock (NVML, read-only), else the B200's 1965 MHz."""
        try:
            import pynvml

            pynvml.nvmlInit()
            return 1e6 * pynvml.nvmlDeviceGetMaxClockInfo(pynvml.nvmlDeviceGetHandleByIndex(index),
                                                          pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            return 1.965e9

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "note": getattr(self, "error", "no samples")}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def cpu_baseline(target_s=12.0, steps=1):
    """Time the C oracle (fwd + bwd + Adam) on a slice of whole groups of this workload."""
    from granulelayer_b200.layout import SparseLayout, init_parameters
    from oracle import oracle as O

    cores = os.cpu_count() or 1
    threads = max(1, min(cores, int(2e9 // (B * D * 8))))
    n_g = N // G

    def run(groups):
        L = SparseLayout(D, n_g * groups, groups, 8, 8, False)
        idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=2, bias_std=0.1)
        if INDEX_RULE == "uniform":
            uniform_indices_(idx, 1002)
        gen = torch.Generator().manual_seed(5)
        x = torch.randn(B, D, generator=gen).numpy()
        dy = torch.randn(B, groups, generator=gen).numpy()
        c = L.counts_tensor("cpu").numpy()
        idx, w, b = idx.numpy(), w.numpy(), b.numpy()
        t0 = time.perf_counter()
        for _ in range(steps):
            O.forward(x, idx, w, b, c, "mean", "relu", threads)
            _, dw, db = O.backward(x, idx, w, b, c, dy, "mean", "relu", threads)
            O.adam_step(w.ravel(), dw.ravel(), np.zeros(w.size), np.zeros(w.size), 1e-3, 0.9, 0.999, 1e-8, 0.0, 1)
            O.adam_step(b.ravel(), db.ravel(), np.zeros(b.size), np.zeros(b.size), 1e-3, 0.9, 0.999, 1e-8, 0.0, 1)
        return (time.perf_counter() - t0) / steps

    t1 = run(1)
    groups = int(max(1, min(64, target_s / max(t1, 1e-3))))
    dt = run(groups) if groups > 1 else t1
    value = B * n_g * groups / dt
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{groups} of {G} groups (x{n_g} neurons) x {B} tokens of this workload, fwd+bwd+Adam, "
                      f"float64 C oracle, {threads} threads of {cores} host CPUs; {dt:.2f} s per step",
            "seconds_per_sample": dt}


def run_reference(args, rank, world):
    if rank != 0:
        return
    cb = cpu_baseline(target_s=args.ref_seconds, steps=1)
    groups = int(cb["sample"].split(" of ")[0])
    from granulelayer_b200.layout import SparseLayout, init_parameters
    from oracle import oracle as O

    n_g = N // G
    L = SparseLayout(D, n_g * groups, groups, 8, 8, False)
    idx, w, b = init_parameters(L, "cpu", dtype=torch.float32, seed=2, bias_std=0.1)
    if INDEX_RULE == "uniform":
        uniform_indices_(idx, 1002)
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(B, D, generator=gen).numpy()
    dy = torch.randn(B, groups, generator=gen).numpy()
    c = L.counts_tensor("cpu").numpy()
    idx, w, b = idx.numpy(), w.numpy(), b.numpy()
    threads = cb["cores"]
    mw, vw, mb, vb = np.zeros(w.size), np.zeros(w.size), np.zeros(b.size), np.zeros(b.size)
    wf, bf = w.ravel().astype(np.float64), b.ravel().astype(np.float64)
    times = []
    for s in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        O.forward(x, idx, w, b, c, "mean", "relu", threads)
        _, dw, db = O.backward(x, idx, w, b, c, dy, "mean", "relu", threads)
        wf, mw, vw = O.adam_step(wf, dw.ravel(), mw, vw, 1e-3, 0.9, 0.999, 1e-8, 0.0, s + 1)
        bf, mb, vb = O.adam_step(bf, db.ravel(), mb, vb, 1e-3, 0.9, 0.999, 1e-8, 0.0, s + 1)
        w, b = wf.reshape(w.shape).astype(np.float32), bf.reshape(b.shape).astype(np.float32)
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = B * n_g * groups / dt
    own = reference_own_cpu()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": config_dict(world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": cb["sample"].split(";")[0]},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_own_cpu": own,
            "note": "reference CPU path = float64 C oracle restating the reference's algorithm on a bounded "
                    "slice of whole groups; the reference's own PyTorch path materialises [B, H] and is timed "
                    "beside it on one whole group (reference_own_cpu)"}
    print(json.dumps(line), flush=True)


REF_DIR = ROOT / "baseline" / "_ref"


def reference_own_cpu(target_s=10.0):
    """The reference's own CPU path on this host, timed beside the port: its materialising PyTorch model
    (reference/pytorch_reference.py reference_forward, fp32) with torch.autograd for dX / dW / db and its
    Adam update (optim.py:39-42, fp32 torch ops), on whole groups of this workload at the full batch, all
    host threads; scaled to neuron-samples/s.  None when the reference is not placed in baseline/_ref."""
    if not (REF_DIR / "sparse_pooling" / "__init__.py").exists():
        return None
    sys.path.insert(0, str(REF_DIR))
    try:
        from sparse_pooling.config import PoolingConfig as RefCfg
        from sparse_pooling.layout import SparseLayout as RefLayout
        from sparse_pooling.layout import init_parameters as ref_init
        from sparse_pooling.reference.pytorch_reference import reference_forward
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"}
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    n_g = N // G
    L = RefLayout(D, n_g, 1, 8, 8, False)
    idx, w, b = ref_init(L, "cpu", dtype=torch.float32, seed=2, bias_std=0.1)
    w, b = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    cfg = RefCfg.parse("mean")
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(B, D, generator=gen).requires_grad_(True)
    dy = torch.randn(B, 1, generator=gen)
    m = [torch.zeros_like(w), torch.zeros_like(b)]
    v = [torch.zeros_like(w), torch.zeros_like(b)]
    times = []
    t_end = time.perf_counter() + target_s
    step = 0
    while step < 2 or (time.perf_counter() < t_end and step < 20):
        t0 = time.perf_counter()
        y = reference_forward(x, idx, w, b, L, cfg)
        (y * dy).sum().backward()
        step += 1
        with torch.no_grad():
            for i, p_ in enumerate((w, b)):
                g_ = p_.grad
                m[i].mul_(0.9).add_(g_, alpha=0.1)
                v[i].mul_(0.999).addcmul_(g_, g_, value=0.001)
                p_.sub_(1e-3 * (m[i] / (1 - 0.9 ** step)) / ((v[i] / (1 - 0.999 ** step)).sqrt() + 1e-8))
                p_.grad = None
        x.grad = None
        if step > 1:
            times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    return {"value": B * n_g / dt, "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"1 of {G} groups ({n_g} neurons) x {B} tokens: the reference's reference_forward + "
                      f"torch.autograd + its Adam update in fp32 torch ops, {cores} threads; {dt:.2f} s per step, "
                      f"{len(times)} timed steps"}


def run_reference_gpu_cover16(args):
    """The reference's Cover-TopK/16 layer (its BF16 kgen K16 kernels) at BASELINE config 4, built its own
    way (experimental/kgen_layout.init_parameters, CoverTopK16Layer.from_envelope), fwd + bwd per step as
    --workload cover16 times ours; rank 0, 1 GPU, comparator only."""
    from sparse_pooling.cover_topk16 import CoverTopK16Layer as RefCT
    from sparse_pooling.experimental.kgen_layout import KLayout as RefKL
    from sparse_pooling.experimental.kgen_layout import init_parameters as ref_init
    from sparse_pooling.supergroups import ConnectivityPlan as RefCP

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Dc, Gc, Bc = 4096, args.cover_outputs, 512
    Hc = Gc * 24576
    w64, b64 = ref_init(RefKL(Dc, Hc, Gc, 64, 256), dev, dtype=torch.bfloat16, seed=3)
    lay = RefCT.from_envelope(w64, b64, input_dim=Dc, hidden_dim=Hc, output_dim=Gc, connectivity=RefCP(64, 64, seed=3),
                              device=dev)
    del w64, b64
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(Bc, Dc, device=dev, generator=gen).to(torch.bfloat16)
    dy = torch.randn(Bc, Gc, device=dev, generator=gen)
    evs = []

    def step(record):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
        if e:
            e[0].record()
        y = lay(x.detach().requires_grad_(True))
        if e:
            e[1].record()
        y.backward(dy.to(y.dtype))
        if e:
            e[2].record()
            evs.append(e)
        for prm in lay.parameters():
            prm.grad = None

    with ClockSampler(dev.index) as clk:
        for _ in range(max(3, args.warmup)):
            step(False)
        torch.cuda.synchronize(dev)
        steps = max(1, args.steps)
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(steps):
            step(True)
        e_ev.record()
        torch.cuda.synchronize(dev)
    ms = s_ev.elapsed_time(e_ev) / steps
    line = {"impl": "reference-gpu", "metric": COVER_METRIC, "value": Bc * Hc / (ms / 1e3), "unit": UNIT,
            "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
            "data": "synthetic", "device": torch.cuda.get_device_name(dev),
            "config": {"workload": "cover16", "N": Hc, "D": Dc, "G": Gc, "global_batch": Bc},
            "fwd_ms": statistics.mean(a.elapsed_time(b) for a, b, _ in evs),
            "bwd_ms": statistics.mean(b.elapsed_time(c) for _, b, c in evs),
            "last_info": {k: str(v)[:120] for k, v in getattr(lay, "last_info", {}).items()} if hasattr(lay, "last_info")
            else None, "clocks": clk.summary(),
            "note": "the reference's own BF16 K16 kernels (not a B200 build of this repository); comparator only"}
    print(json.dumps(line), flush=True)


def run_reference_gpu(args):
    """The reference's own GPU path on this GPU, as a comparator (rank 0, 1 GPU): the unmodified
    package placed in baseline/_ref, driven through its public API (SparsePoolingLayer + FusedAdamW),
    timed with the same CUDA-event step protocol as our arm.  ``--workload modeb``: the published
    table's rows (H = 1e8, D = G = 1024, B = 8192, C = 8 / 64, Mean(ReLU) and Max with save_winners,
    the reference's default BF16 parameters, BF16 x as its bench_end_to_end.py feeds, packed storage,
    its default backend: the m16n8k8 BF16 mma.sync CUDA kernels, Triton for the event backward).
    Default workload: the Mode-A fp32 layer of the headline config (its Triton kernels)."""
    if not (REF_DIR / "sparse_pooling" / "__init__.py").exists():
        print(json.dumps({"impl": "reference-gpu", "unavailable": "reference package not placed in baseline/_ref"}))
        return
    if (REF_DIR / "cache").is_dir():
        os.environ.setdefault("SPARSE_POOL_CACHE_DIR", str(REF_DIR / "cache"))   # prebuilt sm_100 libraries
    sys.path.insert(0, str(REF_DIR))
    if args.workload == "cover16":
        run_reference_gpu_cover16(args)
        return
    from sparse_pooling import SparsePoolingLayer as RefLayer
    from sparse_pooling.optim import FusedAdamW as RefAdam

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.workload == "modeb":
        Hm, Dm, Gm, Bm = args.modeb_neurons, 1024, 1024, 8192
        rdt = torch.float32 if args.ref_dtype == "fp32" else torch.bfloat16
        cases = [(pool, C, rdt) for pool, C in (("mean", 8), ("mean", 64), ("max", 8), ("max", 64))]
        metric, steps = MB_METRIC, max(1, min(args.steps, 5))
    elif args.workload == "sets":
        Hm, Dm, Gm, Bm = args.modeb_neurons, 1024, 1024, 8192
        cases = [("mean", 64, torch.bfloat16), ("mean", 8, torch.bfloat16)]
        metric, steps = SETS_METRIC, max(1, min(args.steps, 5))
    else:
        Hm, Dm, Gm, Bm = N, D, G, B
        cases = [("mean", None, torch.float32)]
        metric, steps = METRIC, max(1, min(args.steps, 5))
    rows = []
    with ClockSampler(dev.index) as clk:
        for pool, C, dtype in cases:
            policy = "save_winners" if pool == "max" else "auto"
            extra = {}
            if args.workload == "sets":
                from sparse_pooling.supergroups import ConnectivityPlan as RefConnectivity
                extra["connectivity"] = RefConnectivity(64, 16, seed=0)
            if args.workload == "modeb" and dtype == torch.float32:
                extra["backend"] = "triton"   # its CUDA kernels are BF16-only; fp32 layers run its Triton path
            lay = RefLayer(Dm, Hm, Gm, shared_neurons=C, pooling=pool, dtype=dtype, device=dev, seed=0,
                           checkpoint_policy=policy, **extra)
            lay.enable_main_grad()
            opt = RefAdam([lay.weight, lay.bias], lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                          moments="bf16" if dtype == torch.bfloat16 else "fp32")
            gen = torch.Generator(device=dev).manual_seed(C or 1)
            x = torch.randn(Bm, Dm, device=dev, generator=gen).to(dtype)
            dy = torch.randn(Bm, Gm, device=dev, generator=gen)
            evs = []

            def step(record):
                e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
                if e:
                    e[0].record()
                y = lay(x.detach().requires_grad_(True))
                if e:
                    e[1].record()
                y.backward(dy.to(y.dtype))
                if e:
                    e[2].record()
                    evs.append(e)
                opt.step()

            for _ in range(max(3, args.warmup)):
                step(False)
            torch.cuda.synchronize(dev)
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(steps):
                step(True)
            e_ev.record()
            torch.cuda.synchronize(dev)
            ms = s_ev.elapsed_time(e_ev) / steps
            info = lay.last_info
            rows.append({"pool": pool, "C": C, "params": "bf16" if dtype == torch.bfloat16 else "f32",
                         "steps": steps, "ms_per_step": ms, "neuron_samples_per_s": Bm * Hm / (ms / 1e3),
                         "fwd_ms": statistics.mean(a.elapsed_time(b) for a, b, _ in evs),
                         "bwd_ms": statistics.mean(b.elapsed_time(c) for _, b, c in evs),
                         "forward_backend": info.get("forward_backend"),
                         "backward_backend": info.get("backward_backend"),
                         "published_rtx3090_bf16_ms": MB_PUBLISHED_MS.get((pool, C))})
            del lay, opt
            torch.cuda.empty_cache()
    head = rows[1] if len(rows) > 1 and args.workload == "modeb" else rows[0]
    line = {"impl": "reference-gpu", "metric": metric, "value": head["neuron_samples_per_s"], "unit": UNIT,
            "n_gpus": 1, "steps": head["steps"], "warmup": max(3, args.warmup), "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "data": "synthetic", "device": torch.cuda.get_device_name(dev),
            "config": {"workload": args.workload, "H": Hm, "D": Dm, "G": Gm, "global_batch": Bm},
            "rows": rows, "clocks": clk.summary(),
            "note": "the reference's own GPU kernels (not a B200 build of this repository); comparator only"}
    print(json.dumps(line), flush=True)


COVER_METRIC = "neuron-samples/s fwd+bwd, Cover-TopK16 K16/C16 layer (N=50,331,648, D=4096, G=2048, B=512)"
FP32_FLOP_PER_SM_CLK = 128 * 2     # 128 fp32 FMA lanes per SM


def cover16_cpu_baseline(lay, x, dy, target_s=8.0):
    """The float64 K/C oracle (numpy) on a bounded slice: the first outputs of the layer, full batch."""
    from oracle import kc_oracle

    idx = lay.indices.cpu().numpy()
    w = lay.weight.detach().double().cpu().numpy()
    b = lay.bias.detach().double().cpu().numpy()
    counts = lay.counts.cpu().numpy()
    xs, dys = x.cpu().numpy(), dy.cpu().numpy()
    Bs = 64
    t0 = time.perf_counter()
    kc_oracle.grads(xs[:Bs], idx[:1], w[:1], b[:1], counts[:1], dys[:Bs, :1])
    t1 = max(time.perf_counter() - t0, 1e-3)
    ng = int(max(1, min(lay.layout.groups, target_s / t1)))
    t0 = time.perf_counter()
    kc_oracle.grads(xs[:Bs], idx[:ng], w[:ng], b[:ng], counts[:ng], dys[:Bs, :ng])
    dt = time.perf_counter() - t0
    return {"value": Bs * int(counts[:ng].sum()) / dt, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{ng} outputs x {Bs} tokens (fwd+bwd, float64 numpy, BLAS threads as configured)"}


def bench_cover16(args, world):
    """BASELINE config 4 (module docstring); rank 0 only."""
    from granulelayer_b200 import _native
    from granulelayer_b200.config import PhysicalPlan
    from granulelayer_b200.cover_topk16 import CoverTopK16Layer
    from granulelayer_b200.kgen import KLayout, init_envelope_parameters
    from granulelayer_b200.supergroups import ConnectivityPlan

    Dc, Gc, Bc = 4096, args.cover_outputs, 512
    Hc = Gc * 24576
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    t0 = time.perf_counter()
    w64, b64 = init_envelope_parameters(KLayout(Dc, Hc, Gc, 64, 256), dev, dtype=torch.bfloat16, seed=3)
    pdt = torch.bfloat16 if args.cover_dtype == "bf16" else torch.float32
    plan = PhysicalPlan(grad_precision="split", b200_f32_tensor_cores="off" if args.cover_kernels == "simt" else "auto",
                        b200_tcgen05={"t5": "on", "t5fwd": "fwd", "t5bwd": "bwd"}.get(args.cover_kernels, "off"))
    lay = CoverTopK16Layer.from_envelope(w64, b64, input_dim=Dc, hidden_dim=Hc, output_dim=Gc,
                                         connectivity=ConnectivityPlan(64, 64, seed=3), device=dev, dtype=pdt,
                                         plan=plan)
    del w64, b64
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    build_s = time.perf_counter() - t0
    gen = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(Bc, Dc, device=dev, generator=gen)
    dy = torch.randn(Bc, Gc, device=dev, generator=gen)

    ev = {"fwd": [], "bwd": []}
    orig = {"fwd": _native.k16_fwd, "fwd_t5": _native.k16_fwd_t5, "bwd": _native.k16_bwd, "bwd_t5": _native.k16_bwd_t5}

    def timed(name, slot):
        def wrap(*a, **k):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            r = orig[name](*a, **k)
            e.record()
            ev[slot].append((s, e))
            return r
        return wrap

    def step():
        xin = x.detach().requires_grad_(True)
        lay.weight.grad = lay.bias.grad = None
        lay(xin).backward(dy)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    _native.k16_fwd, _native.k16_fwd_t5 = timed("fwd", "fwd"), timed("fwd_t5", "fwd")
    _native.k16_bwd, _native.k16_bwd_t5 = timed("bwd", "bwd"), timed("bwd_t5", "bwd")
    n0 = _native.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        with ClockSampler(dev.index) as clk:
            start.record()
            for _ in range(args.steps):
                step()
            end.record()
            torch.cuda.synchronize(dev)
    finally:
        _native.k16_fwd, _native.k16_fwd_t5 = orig["fwd"], orig["fwd_t5"]
        _native.k16_bwd, _native.k16_bwd_t5 = orig["bwd"], orig["bwd_t5"]
    launches = _native.launch_count() - n0
    ms = start.elapsed_time(end) / args.steps
    fwd_ms = statistics.mean(s.elapsed_time(e) for s, e in ev["fwd"])
    bwd_ms = statistics.mean(s.elapsed_time(e) for s, e in ev["bwd"])

    e2e = None
    if not args.no_e2e:
        xh = torch.randn(Bc, Dc, generator=torch.Generator().manual_seed(7)).pin_memory()
        dyh = torch.randn(Bc, Gc, generator=torch.Generator().manual_seed(8)).pin_memory()
        yh = torch.empty(Bc, Gc).pin_memory()
        xd, dyd = torch.empty(Bc, Dc, device=dev), torch.empty(Bc, Gc, device=dev)

        def api_step():
            xd.copy_(xh, non_blocking=True)
            dyd.copy_(dyh, non_blocking=True)
            xin = xd.detach().requires_grad_(True)
            lay.weight.grad = lay.bias.grad = None
            y = lay(xin)
            y.backward(dyd)
            yh.copy_(y.detach(), non_blocking=True)

        for _ in range(2):
            api_step()
        torch.cuda.synchronize(dev)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            api_step()
        e2.record()
        torch.cuda.synchronize(dev)
        t2 = s2.elapsed_time(e2) / args.steps
        e2e = {"value": Bc * Hc / (t2 / 1e3), "unit": UNIT, "ms_per_step": t2,
               "h2d_bytes_per_step": (xh.numel() + dyh.numel()) * 4, "d2h_bytes_per_step": yh.numel() * 4}

    cb = None if (args.no_cpu_baseline or world > 1) else cover16_cpu_baseline(lay, x, dy)
    clocks = clk.summary()
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    peak_tflops = sms * FP32_FLOP_PER_SM_CLK * mhz * 1e6 / 1e12
    bwd_flop = 2 * 48 * Hc * Bc     # per neuron and token: 16 FMA for z, 16 for dW, 16 for dX
    fwd_flop = 2 * 16 * Hc * Bc
    achieved = bwd_flop / (bwd_ms * 1e-3) / 1e12
    hbm, hbm_kind = peak_hbm()
    fkern, bkern = lay.last_info.get("forward_kernel"), lay.last_info.get("backward_kernel")
    if lay.tensor_cores:
        # bf16 MMA flops the backward executes: z once, dX and dW from the bf16 terms -- bf16 layer:
        # 1 + 2 + 2 products (dz as hi + lo); fp32 layer: 6 + 6 + 6 (three-term splits, pairs i + j <= 2)
        mma_flop = bwd_flop / 3 * (5 if pdt == torch.bfloat16 else 18)
        tc_peak, tc_kind = peak_bf16()
        roof = {"bound": "tensor", "kernel": bkern, "achieved": mma_flop / (bwd_ms * 1e-3) / 1e12, "peak": tc_peak,
                "unit": "TFLOP/s", "frac": mma_flop / (bwd_ms * 1e-3) / 1e12 / tc_peak,
                "peak_source": f"{tc_kind} dense bf16 (cuBLAS, burst) -- " + (
                    "tcgen05 MMAs over each set's 64 positions: they execute 4x these flops (a record reads 16)"
                    if "t5" in (bkern or "") else "these are mma.sync tiles"),
                "algorithmic_flop_per_launch": mma_flop, "flop_definition": "bf16 MMA flops of the term products",
                "fp32_equivalent_tflops": achieved,
                # mma.sync bf16 -> fp32 peaks at 2048 flop / clk / SM (ncu peak_sustained), a quarter of tcgen05
                "mma_sync_peak_tflops": sms * 2048 * mhz * 1e6 / 1e12,
                "frac_of_mma_sync_peak": mma_flop / (bwd_ms * 1e-3) / (sms * 2048 * mhz * 1e6)}
    else:
        roof = {"bound": "fp32", "kernel": bkern, "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                "frac": achieved / peak_tflops,
                "peak_source": f"nominal fp32 FMA rate: {sms} SMs x 128 lanes x 2 flop at the median "
                               f"sampled SM clock {mhz} MHz",
                "algorithmic_flop_per_launch": bwd_flop}
    wbytes = Hc * (16 * 4 + 4) + (Hc // 16) * 16
    line = {
        "metric": COVER_METRIC, "value": Bc * Hc / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "f32" if pdt == torch.float32 else "bf16", "data": "synthetic",
        "config": {"workload": "Cover-TopK16 opt-in layer, compact K16/C16 execution, fwd+bwd (BASELINE config 4)"
                               + (("; fp32 on the tensor cores (three-term bf16 splits of x, w, dz)" if lay.tensor_cores
                                   else "; fp32 SIMT kernels") if pdt == torch.float32
                                  else "; bf16 parameters on the tensor cores (the reference's arithmetic), not "
                                       "config 4's fp32"),
                   "kernels": [fkern, bkern],
                   "D": Dc, "N": Hc, "G": Gc, "global_batch": Bc, "envelope": "K64/C256, w64 ~ N(0,1/64) BF16",
                   "S": 64, "R": 64, "Q": int(lay.sg_feat.shape[0]), "records_16": int(Hc // 16),
                   "l2": f"weights {Hc * 64 / 1e9:.1f} GB fp32 > L2: streamed from HBM every pass",
                   "build_seconds": build_s},
        "roofline": dict(roof, hbm_fraction_bwd=(2 * wbytes) / (bwd_ms * 1e-3) / (hbm * 1e9),
                         hbm_peak_source=hbm_kind, traffic=None),
        "kernels_ms": {"fwd": fwd_ms, "bwd": bwd_ms,
                       "fwd_tflops": fwd_flop / (fwd_ms * 1e-3) / 1e12, "bwd_tflops": achieved},
        "clocks": clocks, "gpu_launches": launches, "e2e": e2e, "cpu_baseline": cb,
    }
    print(json.dumps(line), flush=True)


FB_METRIC = "neuron-samples/s fwd+bwd @100M fan-in-8, B=256 (D=4096, G=4096)"


def bench_fwdbwd256(args):
    """BASELINE config 2 (module docstring); rank 0 only, 1 GPU.  Two rows: the drop-in
    SparsePoolingLayer (the reference's storage order, the generic kernels) and the training engine's
    single-rank GroupShardedLayer (octet storage, the lane-per-neuron kernels); the line's value is the
    faster one."""
    import torch.distributed as dist

    from granulelayer_b200 import SparsePoolingLayer, _native
    from granulelayer_b200.distributed import GroupShardedLayer

    Bc = 256
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 1000)))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=300), device_id=dev)
    gen = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(Bc, D, device=dev, generator=gen)
    dy = torch.randn(Bc, G, device=dev, generator=gen)
    rows = {}
    for kind in ("layer", "engine"):
        if kind == "layer":
            lay = SparsePoolingLayer(D, N, G, shared_neurons=None, pooling="mean", dtype=torch.float32, device=dev,
                                     seed=1, bias_std=0.1)
            if INDEX_RULE == "uniform":
                uniform_indices_(lay.indices, 1001)
            names = ("fwd", "bwd")
        else:
            lay = shard_layer(D, N, G, dev, seed=1)
            names = ("fwd_octet", "bwd_octet")
        lay.enable_main_grad()
        ev = {"fwd": [], "bwd": []}
        orig = {n: getattr(_native, n) for n in names}

        def timed(fn, slot):
            def wrap(*a, **k):
                s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_.record()
                fn(*a, **k)
                e_.record()
                ev[slot].append((s_, e_))
            return wrap

        def step():
            lay(x.detach().requires_grad_(True)).backward(dy)

        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize(dev)
        for n, slot in zip(names, ("fwd", "bwd")):
            setattr(_native, n, timed(orig[n], slot))
        n0 = _native.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        try:
            with ClockSampler(dev.index) as clk:
                start.record()
                for _ in range(args.steps):
                    step()
                end.record()
                torch.cuda.synchronize(dev)
        finally:
            for n in names:
                setattr(_native, n, orig[n])
        rows[kind] = {"ms": start.elapsed_time(end) / args.steps,
                      "fwd_ms": statistics.mean(a.elapsed_time(b) for a, b in ev["fwd"]),
                      "bwd_ms": statistics.mean(a.elapsed_time(b) for a, b in ev["bwd"]),
                      "kernels": names, "launches": _native.launch_count() - n0, "clocks": clk.summary()}
        del lay
        torch.cuda.empty_cache()
    head_kind = min(rows, key=lambda k: rows[k]["ms"])
    head = rows[head_kind]
    ms, fwd_ms, bwd_ms = head["ms"], head["fwd_ms"], head["bwd_ms"]
    peak, peak_kind = peak_hbm()
    pass_bytes = param_bytes(N) + gather_bytes(Bc, N)
    achieved = pass_bytes / (bwd_ms * 1e-3) / 1e9
    line = {
        "metric": FB_METRIC, "value": Bc * N / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "100M-neuron fan-in-8 Mode-A fp32 mean-ReLU layer, fwd+bwd at B=256 "
                               "(BASELINE config 2)", "D": D, "N": N, "G": G, "global_batch": Bc, "seed": 1,
                   "bias_std": 0.1, "l2": "parameters (5.2 GB) larger than L2", "timed": head_kind},
        "hbm_roofline_step_frac": (2 * pass_bytes / (peak * 1e9)) / (ms / 1e3),
        "fwd_hbm_roofline_frac": (pass_bytes / (peak * 1e9)) / (fwd_ms / 1e3),
        "roofline": {"bound": "hbm", "kernel": "gl_" + head["kernels"][1] + "_f32", "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                     "traffic": None, "algorithmic_bytes_per_launch": pass_bytes},
        "kernels_ms": {"fwd": fwd_ms, "bwd": bwd_ms}, "clocks": head["clocks"], "gpu_launches": head["launches"],
        "rows": rows,
    }
    print(json.dumps(line), flush=True)
    dist.destroy_process_group()


MB_METRIC = "neuron-samples/s fwd+bwd+opt, Mode B C=64, H=1e8, D=G=1024, B=8192"
MB_PUBLISHED_MS = {("mean", 8): 4898.4, ("mean", 64): 2360.8,   # RTX 3090, BF16 (results/TABLES.md:14, 35,
                   ("max", 8): 513.2, ("max", 64): 409.9}      # 8, 29): context only


# (pool, C, reduction, parameter dtype); bf16 fragment-packed mean / max layers run the tensor-core kernels
MB_ROWS = (("mean", 8, "fast", "f32"), ("mean", 64, "fast", "f32"), ("max", 8, "fast", "f32"), ("max", 64, "fast", "f32"),
           ("mean", 8, "deterministic", "f32"), ("mean", 64, "deterministic", "f32"), ("mean", 8, "fast", "bf16"),
           ("mean", 64, "fast", "bf16"), ("max", 8, "fast", "bf16"), ("max", 64, "fast", "bf16"))


def bench_modeb(args):
    """Mode-B step at the published table's configuration (module docstring); rank 0 only."""
    from granulelayer_b200 import FusedAdamW, PhysicalPlan, SparsePoolingLayer, _native

    Hm, Dm, Gm, Bm = args.modeb_neurons, 1024, 1024, 8192
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows = []
    launches = 0
    with ClockSampler(dev.index) as clk:
        for pool, C, red, dt in MB_ROWS:
            if args.modeb_params and dt not in args.modeb_params.split(","):
                continue
            pooling = pool   # the operators' default activations: Mean(ReLU), Max(identity)
            dtype = torch.bfloat16 if dt == "bf16" else torch.float32
            lay = SparsePoolingLayer(Dm, Hm, Gm, shared_neurons=C, pooling=pooling, dtype=dtype, device=dev,
                                     seed=0, weight_layout="packed", plan=PhysicalPlan(reduction=red))
            lay.enable_main_grad()
            # fp32 layers: fp32 moments; bf16 layers: the reference's optimizer defaults (bf16 moments,
            # stochastic rounding of the parameters)
            opt = FusedAdamW([lay.weight, lay.bias], lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                             moments="fp32" if dt == "f32" else "bf16")
            gen = torch.Generator(device=dev).manual_seed(C)
            x = torch.randn(Bm, Dm, device=dev, generator=gen)
            dy = torch.randn(Bm, Gm, device=dev, generator=gen)
            ev = {"fwd": [], "bwd": []}
            tc = lay._runtime().tensor_cores
            bwd_name = "bwd_events" if pool == "max" else ("bwd_shared_det" if red == "deterministic" else
                                                            "bwd_shared_tc" if tc else "bwd_shared")
            fwd_name = "fwd_shared_tc" if tc else "fwd_shared"
            orig = {"fwd": getattr(_native, fwd_name), "bwd": getattr(_native, bwd_name)}

            def timed(name):
                def wrap(*a, **k):
                    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s_.record()
                    orig[name](*a, **k)
                    e_.record()
                    ev[name].append((s_, e_))
                return wrap

            def step():
                lay(x.detach().requires_grad_(True)).backward(dy)
                opt.step()

            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize(dev)
            setattr(_native, fwd_name, timed("fwd"))
            setattr(_native, bwd_name, timed("bwd"))
            n0 = _native.launch_count()
            steps = max(1, min(args.steps, 5))
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            try:
                s_ev.record()
                for _ in range(steps):
                    step()
                e_ev.record()
                torch.cuda.synchronize(dev)
            finally:
                setattr(_native, fwd_name, orig["fwd"])
                setattr(_native, bwd_name, orig["bwd"])
            launches += _native.launch_count() - n0
            ms = s_ev.elapsed_time(e_ev) / steps
            rows.append({"pool": pool, "C": C, "reduction": red, "params": dt, "forward": fwd_name, "backward": bwd_name,
                         "steps": steps, "ms_per_step": ms,
                         "neuron_samples_per_s": Bm * Hm / (ms / 1e3),
                         "fwd_ms": statistics.mean(a.elapsed_time(b) for a, b in ev["fwd"]),
                         "bwd_ms": statistics.mean(a.elapsed_time(b) for a, b in ev["bwd"]),
                         "fwd_tflops": 2 * 8 * Hm * Bm / (statistics.mean(a.elapsed_time(b) for a, b in ev["fwd"])
                                                          * 1e-3) / 1e12,
                         "published_rtx3090_bf16_ms": MB_PUBLISHED_MS[(pool, C)] if red == "fast" else None})
            if dt == "bf16":
                rows[-1]["published_rtx3090_bf16_ms"] = MB_PUBLISHED_MS[(pool, C)]
            del lay, opt
            torch.cuda.empty_cache()
    head = next((r for r in rows if r["pool"] == "mean" and r["C"] == 64 and r["reduction"] == "fast"
                 and r["params"] == "f32"), rows[0])
    line = {
        "metric": MB_METRIC, "value": head["neuron_samples_per_s"], "unit": UNIT, "n_gpus": 1,
        "steps": head["steps"], "warmup": max(3, args.warmup), "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "Mode B (shared index records), Mean(ReLU) and Max, fwd+bwd+fused Adam, "
                               "fragment-packed storage, fp32 (the reference's published table runs BF16 on an "
                               "RTX 3090)", "H": Hm, "D": Dm, "G": Gm, "global_batch": Bm, "C": [8, 64]},
        "rows": rows, "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)


SETS_METRIC = "neuron-samples/s fwd+bwd+opt, Mode B C=64 with input supergroups S=64 R=16, H=1e8, D=G=1024, B=8192"


def bench_sets(args):
    """bf16 Mode-B layers with input-supergroup connectivity at the reference's supergroup benchmark
    configuration (its bench_supergroups.py defaults: H = 1e8, D = G = 1024, B = 8192, S = 64, R = 16),
    C = 64 and C = 8, Mean(ReLU), fwd + bwd + fused Adam (bf16 moments): the input-set backward
    (gl_bwd_shared_tc_sets) against the generic tensor-core backward on the same layer."""
    from granulelayer_b200 import FusedAdamW, PhysicalPlan, SparsePoolingLayer, _native
    from granulelayer_b200.supergroups import ConnectivityPlan

    Hm, Gm, Bm = args.modeb_neurons, 1024, 8192
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows, launches = [], 0
    # (C, D, S, R): the reference's supergroup benchmark configuration at C = 64 and 8, and a large-D layer
    # where only the input-set kernel's tiles fit
    with ClockSampler(dev.index) as clk:
        for C, Dm, S, R in ((64, 1024, 64, 16), (8, 1024, 64, 16), (64, 4096, 256, 4)):
            lay = SparsePoolingLayer(Dm, Hm, Gm, shared_neurons=C, pooling="mean", dtype=torch.bfloat16, device=dev,
                                     seed=0, weight_layout="packed", connectivity=ConnectivityPlan(S, R, seed=0))
            lay.enable_main_grad()
            opt = FusedAdamW([lay.weight, lay.bias], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, moments="bf16")
            gen = torch.Generator(device=dev).manual_seed(C)
            x = torch.randn(Bm, Dm, device=dev, generator=gen)
            dy = torch.randn(Bm, Gm, device=dev, generator=gen)
            variants = [("grouped", int(t)) for t in args.sets_tokens.split(",")] + [("generic", 0)]
            for variant, tok in variants:
                lay.plan = PhysicalPlan(cuda_input_supergroup_backend=variant, b200_dx_tokens=tok)
                evs = []

                def step(record):
                    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
                    if e:
                        e[0].record()
                    y = lay(x.detach().requires_grad_(True))
                    if e:
                        e[1].record()
                    y.backward(dy)
                    if e:
                        e[2].record()
                        evs.append(e)
                    opt.step()

                for _ in range(max(3, args.warmup)):
                    step(False)
                torch.cuda.synchronize(dev)
                n0 = _native.launch_count()
                steps = max(1, min(args.steps, 5))
                s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s_ev.record()
                for _ in range(steps):
                    step(True)
                e_ev.record()
                torch.cuda.synchronize(dev)
                launches += _native.launch_count() - n0
                ms = s_ev.elapsed_time(e_ev) / steps
                rows.append({"C": C, "D": Dm, "S": S, "R": R, "variant": variant, "tokens": tok or "auto",
                             "backward_kernel": lay.last_info.get("backward_kernel"),
                             "steps": steps, "ms_per_step": ms, "neuron_samples_per_s": Bm * Hm / (ms / 1e3),
                             "fwd_ms": statistics.mean(a.elapsed_time(b) for a, b, _ in evs),
                             "bwd_ms": statistics.mean(b.elapsed_time(c) for _, b, c in evs)})
            del lay, opt
            torch.cuda.empty_cache()
    head = rows[0]
    line = {"metric": SETS_METRIC, "value": head["neuron_samples_per_s"], "unit": UNIT, "n_gpus": 1,
            "steps": head["steps"], "warmup": max(3, args.warmup), "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "bf16 Mode-B Mean(ReLU) layers with input-supergroup connectivity, "
                                   "fwd+bwd+fused Adam", "H": Hm, "G": Gm, "global_batch": Bm,
                       "rows": "(C, D, S, R) = (64, 1024, 64, 16), (8, 1024, 64, 16), (64, 4096, 256, 4)"},
            "rows": rows, "clocks": clk.summary(), "gpu_launches": launches}
    print(json.dumps(line), flush=True)


LOC_METRIC = ("neuron-samples/s fwd+bwd at B=1024, windowed indices, locality/batch sweep "
              "(D=16384, N=100,663,296, G=8192)")


def bench_locality(args):
    """BASELINE config 5 (module docstring); rank 0 only, 1 GPU."""
    from granulelayer_b200 import SparsePoolingLayer, _native
    from granulelayer_b200.layout import windowed_indices

    Dl, Nl, Gl = 16384, 100_663_296, 8192
    batches = [int(v) for v in args.batches.split(",") if v]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lay = SparsePoolingLayer(Dl, Nl, Gl, shared_neurons=None, pooling="mean", dtype=torch.float32, device=dev,
                             seed=4)
    lay.enable_main_grad()
    uniform = lay.indices.clone()
    windowed = windowed_indices(lay.layout, dev, window=512, supergroup=4096, seed=4)
    gen = torch.Generator(device=dev).manual_seed(4)
    rows = []
    launches = 0
    with ClockSampler(dev.index) as clk:
        for mode, idx in (("uniform", uniform), ("windowed", windowed)):
            with torch.no_grad():
                lay.indices.copy_(idx)
            for Bl in batches:
                x = torch.randn(Bl, Dl, device=dev, generator=gen)
                dy = torch.randn(Bl, Gl, device=dev, generator=gen)
                steps = max(1, min(args.steps, 3 if Bl >= 1024 else args.steps))
                res = {"indices": mode, "batch": Bl, "steps": steps}
                for kind in ("fwd", "fwd+bwd"):
                    def step():
                        if kind == "fwd":
                            with torch.no_grad():
                                lay(x)
                        else:
                            lay(x.detach().requires_grad_(True)).backward(dy)
                    for _ in range(max(3, args.warmup)):
                        step()
                    torch.cuda.synchronize(dev)
                    n0 = _native.launch_count()
                    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s_ev.record()
                    for _ in range(steps):
                        step()
                    e_ev.record()
                    torch.cuda.synchronize(dev)
                    launches += _native.launch_count() - n0
                    ms = s_ev.elapsed_time(e_ev) / steps
                    res[kind] = {"ms": ms, "neuron_samples_per_s": Bl * Nl / (ms / 1e3)}
                rows.append(res)
                print(json.dumps({"locality_row": res}), file=sys.stderr, flush=True)
    head = next((r for r in rows if r["indices"] == "windowed" and r["batch"] == 1024), rows[-1])
    hbm, hbm_kind = peak_hbm()
    step_bytes = 2 * param_bytes(Nl) + 2 * gather_bytes(head["batch"], Nl)
    line = {
        "metric": LOC_METRIC, "value": head["fwd+bwd"]["neuron_samples_per_s"], "unit": UNIT, "n_gpus": 1,
        "steps": head["steps"], "warmup": max(3, args.warmup), "ms_per_step": head["fwd+bwd"]["ms"],
        "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "locality/batch sweep, Mode-A fan-in-8 mean-ReLU layer, fwd and fwd+bwd "
                               "(BASELINE config 5)", "D": Dl, "N": Nl, "G": Gl, "batches": batches,
                   "windowed": "supergroups of 4096 neurons, 512-wide random windows, seed 4",
                   "l2": "parameters (5.2 GB) larger than L2"},
        "hbm_roofline_step_frac": (step_bytes / (hbm * 1e9)) / (head["fwd+bwd"]["ms"] / 1e3),
        "sweep": rows, "clocks": clk.summary(), "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)


def main():
    global N, G, INDEX_RULE
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-seconds", type=float, default=4.0)
    ap.add_argument("--workload", default="layer100m",
                    choices=["layer100m", "fwdbwd256", "cover16", "locality", "modeb", "sets"])
    ap.add_argument("--batches", default="1,32,256,1024,4096", help="locality: batch sizes of the sweep")
    ap.add_argument("--modeb-neurons", type=int, default=100_000_000,
                    help="modeb: neurons (default 1e8 = the published table; fewer for ncu captures)")
    ap.add_argument("--modeb-params", default="", help="modeb: only the rows of these parameter dtypes "
                                                       "(comma list of f32, bf16; default all)")
    ap.add_argument("--sets-tokens", default="0", help="sets: token tiles of the input-set backward to time "
                                                      "(comma list; 0 = automatic)")
    ap.add_argument("--ref-dtype", default="bf16", choices=["fp32", "bf16"],
                    help="--impl reference-gpu --workload modeb: the reference layer's parameter dtype")
    ap.add_argument("--cover-dtype", default="fp32", choices=["fp32", "bf16"],
                    help="cover16: parameter storage (fp32 = config 4; bf16 = the reference's, on the tensor cores)")
    ap.add_argument("--cover-kernels", default="tc", choices=["tc", "t5", "t5fwd", "t5bwd", "simt"],
                    help="cover16: mma.sync tensor-core kernels (default); t5 = forward and backward on tcgen05 "
                         "(TMEM), t5fwd / t5bwd = one of them; simt = the fp32 SIMT kernels (fp32 parameters)")
    ap.add_argument("--cover-outputs", type=int, default=2048,
                    help="cover16: outputs of 24,576 neurons (default 2048 = config 4; fewer for ncu captures)")
    ap.add_argument("--index-rule", default=INDEX_RULE, choices=sorted(INDEX_RULES),
                    help="layer100m / fwdbwd256: the reference's distinct-sorted init, or the configs' uniform "
                         "rule with replacement")
    ap.add_argument("--groups", type=int, default=G,
                    help="pooling groups of 24,576 neurons (default 4096 = the full 100M layer; smaller values "
                         "give the reduced cases used for ncu captures)")
    args = ap.parse_args()
    INDEX_RULE = args.index_rule
    if args.groups != G:
        N, G = args.groups * (N // G), args.groups
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference-gpu":
        if rank == 0:
            run_reference_gpu(args)
        return
    if args.workload == "cover16":
        if rank == 0:
            bench_cover16(args, world)
        return
    if args.workload == "locality":
        if rank == 0:
            bench_locality(args)
        return
    if args.workload == "fwdbwd256":
        if rank == 0:
            bench_fwdbwd256(args)
        return
    if args.workload == "modeb":
        if rank == 0:
            bench_modeb(args)
        return
    if args.workload == "sets":
        if rank == 0:
            bench_sets(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch.distributed as dist

    from granulelayer_b200 import FusedAdamW, SparsePoolingLayer, _native
    from granulelayer_b200.distributed import GroupShardedLayer, ShardedTrainStep

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 or "MASTER_ADDR" in os.environ:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 1000)))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=300), device_id=dev)

    lay = shard_layer(D, N, G, dev, seed=2)
    opt = FusedAdamW([lay.weight, lay.bias], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, moments="fp32")
    trainer = ShardedTrainStep(lay, opt)
    n_local = int(lay.counts.sum())
    gen = torch.Generator(device=dev).manual_seed(1234)
    x = torch.randn(B, D, device=dev, generator=gen)
    dy = torch.randn(B, G, device=dev, generator=gen)
    rt = lay.runtime()

    # per-kernel timing: events around the forward and backward launches on their stream
    ev = {"fwd": [], "bwd": []}
    orig_fwd, orig_bwd = rt.forward, rt.backward

    def timed(name, fn):
        def wrap(*a, **k):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*a, **k)
            e.record()
            ev[name].append((s, e))
            return out
        return wrap

    for _ in range(args.warmup):
        trainer.step(x, dy)
    torch.cuda.synchronize(dev)
    rt.forward, rt.backward = timed("fwd", orig_fwd), timed("bwd", orig_bwd)
    dist.barrier()
    torch.cuda.synchronize(dev)
    n0 = _native.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        start.record()
        for _ in range(args.steps):
            trainer.step(x, dy)
        end.record()
        torch.cuda.synchronize(dev)
    dist.barrier()
    launches = _native.launch_count() - n0
    rt.forward, rt.backward = orig_fwd, orig_bwd
    ms_local = start.elapsed_time(end) / args.steps
    fwd_ms = statistics.mean(s.elapsed_time(e) for s, e in ev["fwd"])
    bwd_ms = statistics.mean(s.elapsed_time(e) for s, e in ev["bwd"])
    t = torch.tensor([ms_local, fwd_ms, bwd_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_max, bwd_max = t.tolist()

    # end to end through the public API: pinned host buffers in, pooled output out, every step
    e2e = None
    if not args.no_e2e:
        xh = torch.randn(B, D, generator=torch.Generator().manual_seed(7)).pin_memory()
        dyh = torch.randn(B, G, generator=torch.Generator().manual_seed(8)).pin_memory()
        yh = torch.empty(B, G).pin_memory()
        xd = torch.empty(B, D, device=dev)
        dyd = torch.empty(B, G, device=dev)

        def api_step():
            xd.copy_(xh, non_blocking=True)
            dyd.copy_(dyh, non_blocking=True)
            xin = xd.detach().requires_grad_(True)
            y = lay(xin)
            y.backward(dyd)
            opt.step()
            yh.copy_(y.detach(), non_blocking=True)

        for _ in range(2):
            api_step()
        torch.cuda.synchronize(dev)
        dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            api_step()
        e2.record()
        torch.cuda.synchronize(dev)
        t2 = torch.tensor([s2.elapsed_time(e2) / args.steps], device=dev)
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e = {"value": B * N / (t2.item() / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": xh.numel() * 4 + dyh.numel() * 4, "d2h_bytes_per_step": yh.numel() * 4,
               "ms_per_step": t2.item()}

    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
        cb.pop("seconds_per_sample", None)

    if rank == 0:
        peak, peak_kind = peak_hbm()
        bwd_bytes = param_bytes(n_local) + gather_bytes(B, n_local)
        achieved = bwd_bytes / (bwd_ms * 1e-3) / 1e9
        step_bytes = 2 * param_bytes(N) + 2 * gather_bytes(B, N)
        traffic = BWD_DRAM_BYTES_PER_NEURON * n_local if B == 1024 else None
        # physical limiter: the shared-memory data path.  Per (neuron, input, 4 tokens) the backward moves a
        # 16-byte x gather and a 16-byte dX scatter through it, 128 bytes per SM clock at best.
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        smem_floor_ms = (B * n_local * K_FAN * 8) / (128 * sms * ClockSampler.max_clock_hz(dev.index)) * 1e3
        line = {
            "metric": METRIC, "value": B * N / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_dict(world),
            "hbm_roofline_step_frac": (step_bytes / (peak * 1e9)) / (ms / 1e3),
            "roofline": {"bound": "hbm", "kernel": rt.last_info.get("backward_kernel", "gl_bwd_f32"),
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic,
                         "traffic_source": f"ncu dram bytes of a 512-group capture, scaled by neuron count "
                                           f"({BWD_PROFILE})",
                         "algorithmic_bytes_per_launch": bwd_bytes,
                         "definition": "(param + x-gather bytes) per launch / CUDA-event launch time; "
                                       "gathers count as logical HBM bytes per the baseline definition, "
                                       "although they are served from shared memory",
                         "smem_floor_ms": smem_floor_ms, "smem_floor_frac": smem_floor_ms / bwd_ms,
                         "smem_floor_definition": "B*N*8 x (16-byte gather + 16-byte scatter) / 4 tokens, at "
                                                  "128 bytes per SM clock, all SMs at the maximum SM clock"},
            "kernels_ms": {"fwd": fwd_ms, "bwd": bwd_ms, "fwd_max_rank": fwd_max, "bwd_max_rank": bwd_max},
            "clocks": clk.summary(), "gpu_launches": launches,
            "e2e": e2e, "cpu_baseline": cb,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
