#!/usr/bin/env python
"""Benchmark of the COAT quantization hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Headline workload ("step"): one fused FP8-AdamW step with Dynamic Range Expansion over the full
Llama-2-7B parameter set (291 tensors, 6 738 415 616 fp32 master weights, synthetic N(0,1e-3)
gradients, E4M3 moments in groups of 128), sharded ZeRO-style over the N GPUs on 128-element
boundaries and followed by the all-gather of the updated bf16 weights.  Total work is fixed, so
scaling is "strong".  Rank 0 prints ONE JSON line.

`--impl reference` times the reference's optimizer step on the host cores, on a bounded sample of the same
workload: the C restatement of its kernel (oracle/, OpenMP over groups, every core the process may use) as the
line's value, and beside it the reference's pure-PyTorch path (oracle/adamw_torch.py).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fp8_adamw_expand_params_per_s"
UNIT = "params/s"
BYTES_PER_PARAM = 16.375      # read p4 g4 m1 v1, write p4 m1 v1, 12 fp32 per 128-group
BYTES_PER_PARAM_BF16 = 18.375  # + the bf16 weight copy for the all-gather
HYPER = dict(lr=1e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)


def llama2_7b_shapes():
    H, I, V, L = 4096, 11008, 32000, 32
    layer = [(H, H)] * 4 + [(I, H), (I, H), (H, I), (H,), (H,)]
    return [(V, H)] + layer * L + [(H,), (V, H)]


def numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, col in (("hw_slowdown", 5), ("hw_thermal_slowdown", 6), ("sw_thermal_slowdown", 7),
                              ("sw_power_cap", 8)):
                if r[col].lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the C restatement of the reference kernel on the host cores
# ------------------------------------------------------------------------------------------------

def host_cores():
    """Cores this process may run on (not the machine's count: a container or a launcher may have cut it down)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_steps(n_params, min_seconds, min_steps=2, seed=0):
    """Time oracle.fp8_adamw_expand_step on `n_params` fp32 params; returns (params/s, steps, seconds, threads).
    The OpenMP thread count is set explicitly (torch.distributed.run exports OMP_NUM_THREADS=1) and the count in
    effect is what is reported."""
    import torch
    from oracle import adamw as O
    threads = O.set_num_threads(host_cores())
    gen = torch.Generator().manual_seed(seed)
    G = (n_params + 127) // 128
    p = torch.randn(n_params, generator=gen) * 0.02
    g = torch.randn(n_params, generator=gen) * 1e-3
    m = torch.zeros(n_params, dtype=torch.uint8)
    v = torch.zeros(n_params, dtype=torch.uint8)
    vec = [torch.zeros(G), torch.ones(G), torch.ones(G), torch.zeros(G), torch.ones(G), torch.ones(G)]

    def one(step):
        O.fp8_adamw_expand_step(p, g, m, vec[0], vec[1], vec[2], v, vec[3], vec[4], vec[5], HYPER["betas"][0],
                                HYPER["betas"][1], HYPER["lr"], HYPER["weight_decay"], HYPER["eps"], step, 128, 16)

    one(1)  # warm-up: leaves realistic (non-zero) state behind
    steps, t0 = 0, time.perf_counter()
    while steps < min_steps or time.perf_counter() - t0 < min_seconds:
        one(2 + steps)
        steps += 1
    dt = time.perf_counter() - t0
    return n_params * steps / dt, steps, dt, threads


def cpu_pure_pytorch_steps(n_params=4096 * 4096, warmup=1, steps=3, seed=0):
    """The reference's pure-PyTorch FP8AdamW-expand path (its test's expectation, restated in oracle/adamw_torch.py
    and pinned to the reference's own output by the CPU tests) on the host cores: 1 warm-up + 3 timed steps on a
    4096 x 4096 tensor.  Returns {value, unit, cores, kind, sample}."""
    import torch
    from oracle import adamw_torch as T
    threads = host_cores()
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(seed)
    p = torch.randn(n_params, generator=gen) * 0.02
    m = torch.randn(n_params, generator=gen) * 1e-3
    v = (torch.randn(n_params, generator=gen) * 1e-3).square_() + 1e-12
    grads = [torch.randn(n_params, generator=gen) * 1e-3 for _ in range(2)]
    for i in range(warmup):
        T.pure_pytorch_expand_step(p, grads[i & 1], m, v, HYPER["betas"][0], HYPER["betas"][1], HYPER["lr"],
                                   HYPER["weight_decay"], HYPER["eps"], i)
    t0 = time.perf_counter()
    for i in range(steps):
        T.pure_pytorch_expand_step(p, grads[i & 1], m, v, HYPER["betas"][0], HYPER["betas"][1], HYPER["lr"],
                                   HYPER["weight_decay"], HYPER["eps"], warmup + i)
    dt = time.perf_counter() - t0
    return {"value": n_params * steps / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} steps of one 4096x4096 tensor in {dt:.1f} s after {warmup} warm-up: the reference's "
                      "pure-PyTorch path (the expectation of its optimizer test, torch fake-quantizer), restated in "
                      "oracle/adamw_torch.py"}


def workload_config(world, exchange, workload="llama2-7b", note=""):
    """The `config` object of the JSON line; both arms print the same one."""
    what = ("FP8AdamW-expand step over the full Llama-2-7B parameter set (291 tensors, 6738415616 params)"
            if workload == "llama2-7b" else "FP8AdamW-expand step over one 4096x4096 tensor (profiling case)")
    how = {"p2p": " stored by the same kernel into every peer's buffer over NVLink (fused step + all-gather), "
                  "one-element all-reduce as the closing barrier",
           "nccl": " + bucketed NCCL all-gather on a side stream",
           "copy": " + bucketed peer copies (DMA engines) of the bf16 weights on side streams",
           "hybrid": " + bf16 weights to most peers by the step kernel's own bulk stores, to the rest by bucketed peer "
                     "copies (DMA engines) on side streams",
           "auto": " + exchange chosen by world size",
           None: ""}[exchange if world > 1 else None]
    return {"workload": what + ", fp32 master weights, E4M3 moments group 128, bf16 weight copy" + how + note,
            "parallelism": f"zero-shard x{world} on 128-element group boundaries",
            "l2": "inputs larger than L2 (>= 10 GB per GPU per step)" if workload == "llama2-7b" else
                  "inputs larger than L2 (308 MB per step)",
            "hyper": {"lr": 1e-4, "betas": [0.9, 0.95], "wd": 0.1, "eps": 1e-8, "expand_min": 16}}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n = 4096 * 4096
    per_step = []
    for _ in range(max(0, args.warmup)):
        cpu_reference_steps(n, 0.0, min_steps=1)
    cores = 1
    for _ in range(max(1, args.steps)):
        rate, steps, dt, cores = cpu_reference_steps(n, 1.0, min_steps=1)
        per_step.append(dt / steps)
    ms = 1e3 * sum(per_step) / len(per_step)
    value = n / (ms / 1e3)
    sample = ("bounded sample of the workload: one 4096x4096 fp32 tensor (16 777 216 params) per step, C restatement "
              f"of the reference kernel (oracle/fp8_adamw_oracle.c), OpenMP over groups, {cores} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 math / e4m3 state", "data": "synthetic",
        # (the same configuration text as the GPU arm prints: "auto" resolved by the number of GPUs)
        "config": workload_config(args.gpus, ("copy" if args.gpus == 2 else "p2p") if args.exchange == "auto" else args.exchange),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                         "pure_pytorch": cpu_pure_pytorch_steps()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------

# DRAM bytes per parameter of the optimizer kernel, from ncu (dram__bytes_read.sum + dram__bytes_write.sum, one launch):
# at the benchmark's own size, 72.056 GB read + 56.447 GB written for the 6 738 415 616 parameters of one full launch
# (the two counters take a single pass, so the capture holds nothing back and restores nothing); on the 4096x4096
# profiling case, whose 308 MB the 126 MB L2 absorbs in part, 171.2 + 94.1 MB for 16 777 216 parameters
NCU_DRAM_BYTES_PER_PARAM_FULL = (72.055545088e9 + 56.447258112e9) / 6738415616
NCU_DRAM_BYTES_PER_PARAM_C1 = (171.213824e6 + 94.058240e6) / (4096 * 4096)


def fill_synthetic(opt, shapes, torch):
    """p ~ N(0, 0.02), g ~ N(0, 1e-3), seeded per tensor (seed 100+i), generated on the device piece by
    piece (the full set is 27 GB per array; there are no checkpoints or datasets on the box)."""
    gen = torch.Generator(device=opt.device)
    for pc in opt.my_pieces:
        gen.manual_seed(100 + pc.tensor * 16 + opt.rank)
        sl = slice(pc.offset, pc.offset + pc.numel)
        opt.param[sl].normal_(0.0, 0.02, generator=gen)
        opt.grad[sl].normal_(0.0, 1e-3, generator=gen)


def e2e_public_api(torch, device, steps, warmup):
    """params/s through the public optimizer API (CoatAdamW.step) with HOST gradients: every step copies
    the gradients of one Llama-2-7B decoder layer (9 tensors, 202 383 360 params) from pinned host memory
    and reads the updated fp32 weights back to pinned host memory (all of both inside the timed region)."""
    from coat_b200.optimizer import CoatAdamW
    H, I = 4096, 11008
    shapes = [(H, H)] * 4 + [(I, H), (I, H), (H, I), (H,), (H,)]
    gen = torch.Generator().manual_seed(7)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(device)) for s in shapes]
    host_g = [(torch.randn(s, generator=gen) * 1e-3).pin_memory() for s in shapes]
    host_p = [torch.empty(s).pin_memory() for s in shapes]
    for p in params:
        p.grad = torch.empty_like(p)
    opt = CoatAdamW(params, **HYPER)
    n = sum(numel(s) for s in shapes)

    # Three streams: gradients in, step, weights out.  The copy-in of step k+1 and the copy-out of step k both
    # wait only for the kernel of step k, so they share the two directions of the link; the kernel of step k+1
    # waits for both (it overwrites the weights that are being read out and consumes the new gradients).
    s_in, s_step, s_out = (torch.cuda.Stream(device=device) for _ in range(3))
    ev_in, ev_step, ev_out = (torch.cuda.Event() for _ in range(3))
    s_step.wait_stream(torch.cuda.current_stream(device))
    ev_step.record(s_step)
    ev_out.record(s_out)

    def one():
        s_in.wait_event(ev_step)            # the previous step no longer reads the gradient buffers
        with torch.cuda.stream(s_in):
            for p, hg in zip(params, host_g):
                p.grad.copy_(hg, non_blocking=True)
            ev_in.record(s_in)
        s_step.wait_event(ev_in)
        s_step.wait_event(ev_out)           # the previous weights have been read out
        with torch.cuda.stream(s_step):
            opt.step()
            ev_step.record(s_step)
        s_out.wait_event(ev_step)
        with torch.cuda.stream(s_out):
            for p, hp in zip(params, host_p):
                hp.copy_(p.detach(), non_blocking=True)
            ev_out.record(s_out)

    def drain():
        for st in (s_in, s_step, s_out):
            st.synchronize()

    for _ in range(max(warmup, 2)):
        one()
    drain()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(s_step)
    s_in.wait_event(t0)
    for _ in range(steps):
        one()
    s_step.wait_stream(s_out)               # the timed region ends when the last weights have arrived
    t1.record(s_step)
    drain()
    ms = t0.elapsed_time(t1) / steps
    return ms, 4 * n, 4 * n, n


def quantizer_extras(torch, device, peak):
    """GB/s of the quantizers on the activation benchmark tensor (8192 tokens x 4096 bf16,
    0.1 % of the entries x100): algorithmic bytes / CUDA-event time of the C-ABI calls on preallocated
    outputs, 20 calls replayed from one CUDA graph so that host launch overhead (comparable to these
    15-30 us kernels) stays out of the device time.  The input (64 MB) is smaller than L2, so four
    distinct inputs rotate (256 MB of reads between two uses of the same buffer)."""
    from coat_b200 import _lib
    L = _lib.lib()
    M, N = 8192, 4096
    gen = torch.Generator(device=device).manual_seed(1)
    xs = []
    for _ in range(4):
        x = torch.randn(M, N, generator=gen, device=device)
        x = torch.where(torch.rand(M, N, generator=gen, device=device) < 1e-3, x * 100, x).to(torch.bfloat16)
        xs.append(x)
    y = torch.empty(M, N, dtype=torch.uint8, device=device)
    y_t = torch.empty(N, M, dtype=torch.uint8, device=device)
    s_y = torch.empty(M, N // 16, dtype=torch.bfloat16, device=device)
    s_y_t = torch.empty(N, M // 16, dtype=torch.bfloat16, device=device)
    s_max = torch.empty((), dtype=torch.bfloat16, device=device)
    amax = torch.empty(1, dtype=torch.int32, device=device)
    sync_words = torch.zeros(4, dtype=torch.int32, device=device)   # the one-launch kernel's words: zero in, zero out
    E4M3, BF16 = _lib.E4M3, _lib.BF16

    def st():
        return _lib.stream_ptr(device)

    def group(x):
        return L.coat_fp8_quantize(x.data_ptr(), y.data_ptr(), s_y.data_ptr(), M, N, N, 16, E4M3, BF16, BF16, 0, st())

    def pertensor(x, transposed):
        rc = L.coat_fp8_group_scales_amax(x.data_ptr(), None if transposed else s_y.data_ptr(), amax.data_ptr(), M, N,
                                          N, 16, E4M3, BF16, BF16, 0, st())
        return rc or L.coat_fp8_division(x.data_ptr(), y.data_ptr(), y_t.data_ptr() if transposed else None, None,
                                         s_max.data_ptr(), amax.data_ptr(), M, N, N, E4M3, BF16, BF16, 0, st())

    def pertensor_one_launch(x, transposed=False):
        return L.coat_fp8_quantize_pertensor(x.data_ptr(), y.data_ptr(), y_t.data_ptr() if transposed else None,
                                             None if transposed else s_y.data_ptr(), s_max.data_ptr(),
                                             sync_words.data_ptr(), M, N, N, 16, E4M3, BF16, BF16, 0, st())

    def qt(x):
        return L.coat_fp8_quantize_transpose(x.data_ptr(), y.data_ptr(), s_y.data_ptr(), y_t.data_ptr(),
                                             s_y_t.data_ptr(), M, N, N, 16, E4M3, BF16, BF16, 0, st())

    def amax_pass(x):
        return L.coat_fp8_group_scales_amax(x.data_ptr(), None, amax.data_ptr(), M, N, N, 16, E4M3, BF16, BF16, 0, st())

    def division(x, transposed):
        return L.coat_fp8_division(x.data_ptr(), y.data_ptr(), y_t.data_ptr() if transposed else None, None,
                                   s_max.data_ptr(), amax.data_ptr(), M, N, N, E4M3, BF16, BF16, 0, st())

    cases = {
        "quantize_1x16": (group, 3.125, 1),
        "quantize_pertensor": (pertensor_one_launch, 3.125, 1),   # what fp8_quantize_pertensor calls
        "quantize_pertensor_two_launches": (lambda x: pertensor(x, False), 3.125, 2),
        "quantize_pertensor_transpose": (lambda x: pertensor_one_launch(x, True), 4.0, 1),   # what the operator calls
        "quantize_pertensor_transpose_two_launches": (lambda x: pertensor(x, True), 4.0, 2),
        "quantize_transpose_1x16": (qt, 4.25, 1),
        # the two passes of the per-tensor quantizers on their own
        "pass1_tensor_amax": (amax_pass, 2.0, 1),
        "pass2_division": (lambda x: division(x, False), 3.0, 1),
        "pass2_division_transpose": (lambda x: division(x, True), 4.0, 1),
    }
    # yardstick at THIS size: a device-to-device copy that moves as many bytes as the 1x16 quantizer's algorithmic
    # traffic (52 MB read + 52 MB written), in the same harness; the measured-peak denominator comes from a copy
    # hundreds of times larger, which amortises launch and ramp-up
    copy_src = [torch.empty(M * N * 25 // 16, dtype=torch.uint8, device=device) for _ in range(4)]
    copy_dst = torch.empty_like(copy_src[0])
    src_of = {x.data_ptr(): c for x, c in zip(xs, copy_src)}

    def same_size_copy(x):
        copy_dst.copy_(src_of[x.data_ptr()])
        return 0
    cases["copy_of_the_same_bytes_as_quantize_1x16"] = (same_size_copy, 3.125, 1)
    out = {}
    iters = 20
    for name, (fn, bytes_per_elem, launches) in cases.items():
        for i in range(4):
            _lib.check(fn(xs[i]), name)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(iters):
                fn(xs[i & 3])
        for _ in range(25):   # warm-up: a few hundred launches, so that the clocks have ramped up
            graph.replay()
        torch.cuda.synchronize(device)
        times = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize(device)
            times.append(e0.elapsed_time(e1) / iters)
        ms = sorted(times)[len(times) // 2]   # median of 5 replays of 20 calls
        gbs = M * N * bytes_per_elem / (ms / 1e3) / 1e9
        out[name] = {"us": ms * 1e3, "GB/s": gbs, "frac_of_measured_hbm": gbs / peak,
                     "algorithmic_bytes_per_elem": bytes_per_elem, "kernels_per_call": launches}
    return out


def gemm_extras(torch, device, iters=10):
    """TFLOP/s of the FP8 GEMM on the Llama-2-7B MLP shape (8192 tokens, 4096 -> 11008): forward
    (E4M3 x E4M3), dgrad and wgrad (E5M2 x E4M3), 2*M*N*K flops each = 0.7388 TFLOP, CUDA-event time of the
    C-ABI call on preallocated outputs.  Operands (45-90 MB each, > 200 MB per GEMM with the output) exceed
    L2 together.  Fractions are against a dense FP8 rate measured in the same run (fp8_peak_yardstick: the library's
    FP8 GEMM at 8192^3, burst and sustained), against 2x the measured bf16 GEMM peak of this pool and against the
    nominal 4500 dense FP8 TFLOP/s."""
    from coat_b200 import _lib
    L = _lib.lib()
    T, H, I = 8192, 4096, 11008
    gen = torch.Generator(device=device).manual_seed(2)

    def codes(r, c, dtype, scale):
        return (torch.randn(r, c, generator=gen, device=device) * scale).to(dtype)

    x, x_t = codes(T, H, torch.float8_e4m3fn, 50), codes(H, T, torch.float8_e4m3fn, 50)
    w, w_t = codes(I, H, torch.float8_e4m3fn, 50), codes(H, I, torch.float8_e4m3fn, 50)
    g, g_t = codes(T, I, torch.float8_e5m2, 500), codes(I, T, torch.float8_e5m2, 500)
    s = torch.tensor(0.01, dtype=torch.bfloat16, device=device)
    bf16_peak, bf16_sustained = 1651.6, 1393.3
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
            bf16_peak = float(peaks.get("bf16_tflops", bf16_peak))
            bf16_sustained = float(peaks.get("bf16_tflops_sustained", bf16_sustained))
    out = {}
    calls = {}
    yard = fp8_peak_yardstick(torch, device) if iters >= 10 else {"unavailable": "profiling run"}
    time.sleep(0.5)   # let the clocks recover from the yardstick's sustained loop before the bursts
    for name, a, bm in (("forward_e4m3xe4m3", x, w), ("dgrad_e5m2xe4m3", g, w_t), ("wgrad_e5m2xe4m3", g_t, x_t)):
        M, K = a.shape
        N = bm.shape[0]
        c = torch.empty(M, N, dtype=torch.bfloat16, device=device)

        def call(a=a, bm=bm, c=c, M=M, N=N, K=K):
            return L.coat_fp8_gemm(a.data_ptr(), bm.data_ptr(), c.data_ptr(), None, s.data_ptr(), s.data_ptr(), None,
                                   M, N, K, _lib.fp8_enum_of(a), _lib.fp8_enum_of(bm), _lib.BF16, _lib.BF16, 0, 16, 0,
                                   _lib.stream_ptr(device))
        calls[name] = (call, M, N, K)
    # the forward GEMM with the fused 1x16 quantising epilogue (FP8 codes + bf16 group scales instead of bf16), as the
    # gate / up projections of the decoder layer use it
    cq = torch.empty(T, I, dtype=torch.uint8, device=device)
    sq = torch.empty(T, I // 16, dtype=torch.bfloat16, device=device)

    def call_q():
        return L.coat_fp8_gemm(x.data_ptr(), w.data_ptr(), cq.data_ptr(), sq.data_ptr(), s.data_ptr(), s.data_ptr(), None,
                               T, I, H, _lib.E4M3, _lib.E4M3, _lib.BF16, _lib.BF16, 1, 16, 0, _lib.stream_ptr(device))
    calls["forward_e4m3xe4m3_quantising_epilogue_1x16"] = (call_q, T, I, H)

    def timed(call, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            call()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / n

    # bursts of `iters` launches first (clocks still high), then each GEMM back to back for ~0.2 s, where the
    # 1 kW power cap pulls the SM clock down to ~1.3 GHz
    for name, (call, M, N, K) in calls.items():
        for _ in range(3):
            _lib.check(call(), name)
        torch.cuda.synchronize(device)
        ms = timed(call, iters)
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        out[name] = {"M": M, "N": N, "K": K, "us": ms * 1e3, "TFLOP/s": tf, "frac_of_2x_measured_bf16": tf / (2 * bf16_peak),
                     "frac_of_nominal_fp8": tf / 4500.0}
        if "burst_tflops" in yard:
            out[name]["frac_of_measured_fp8_burst"] = tf / yard["burst_tflops"]
        time.sleep(0.05)
    for name, (call, M, N, K) in calls.items():
        if iters < 10:   # profiling runs ask for a few launches only
            continue
        tf_sus = 2.0 * M * N * K / (timed(call, 600) / 1e3) / 1e12
        out[name]["TFLOP/s_sustained"] = tf_sus
        out[name]["frac_of_2x_measured_bf16_sustained"] = tf_sus / (2 * bf16_sustained)
        if "sustained_tflops" in yard:
            out[name]["frac_of_measured_fp8_sustained"] = tf_sus / yard["sustained_tflops"]
    out["fp8_peak_yardstick"] = yard
    out["device_status"] = L.coat_fp8_gemm_device_status()
    return out


def blockscaled_extras(torch, device, peak, iters=10):
    """The DeepSeek-style block-scaled path on the Llama-2-7B MLP forward shape: the 128-granular quantizers
    (GB/s of algorithmic bytes) and the block-scaled GEMM (TFLOP/s), CUDA-event time of the public python calls."""
    from coat_b200.activation.deepseek import gemm_fp8_fp8_bf16_nt
    from coat_b200.activation.real_quantization import fp8_quantize_perblock, fp8_quantize_transpose
    T, H, I = 8192, 4096, 11008
    gen = torch.Generator(device=device).manual_seed(4)
    x = torch.randn(T, H, generator=gen, device=device).to(torch.bfloat16)
    w = (torch.randn(I, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / n

    out = {}
    ms = timed(lambda: fp8_quantize_transpose(x, 128, "E4M3", scale_dtype=torch.float32), iters)
    by = T * H * (2 + 1 + 1 + 8.0 / 128)
    out["quantize_transpose_1x128"] = {"us": ms * 1e3, "GB/s": by / ms / 1e6, "frac_of_measured_hbm": by / ms / 1e6 / peak}
    ms = timed(lambda: fp8_quantize_perblock(w, 128, "E4M3", scale_dtype=torch.float32), iters)
    by = I * H * 3.0
    out["quantize_perblock_128x128"] = {"us": ms * 1e3, "GB/s": by / ms / 1e6, "frac_of_measured_hbm": by / ms / 1e6 / peak}
    (qx, sx), _ = fp8_quantize_transpose(x, 128, "E4M3", scale_dtype=torch.float32)
    sx = sx.t().contiguous().t()
    qw, sw = fp8_quantize_perblock(w, 128, "E4M3", scale_dtype=torch.float32)
    c = torch.empty(T, I, dtype=torch.bfloat16, device=device)
    ms = timed(lambda: gemm_fp8_fp8_bf16_nt((qx, sx), (qw, sw), c), iters)
    tf = 2.0 * T * I * H / (ms / 1e3) / 1e12
    out["gemm_blockscaled_forward"] = {"M": T, "N": I, "K": H, "us": ms * 1e3, "TFLOP/s": tf,
                                       "frac_of_nominal_fp8": tf / 4500.0}
    return out


def layer_extras(torch, device, iters=5, with_reference_operators=False):
    """Forward + backward of ONE Llama-2-7B decoder layer (hidden 4096, 32 heads, MLP 11008) on 4 x 2048 tokens
    through the FP8 layer of this package, and, beside it, the same layer in plain bf16 torch (cuBLAS GEMMs,
    SDPA, eager elementwise ops) as a yardstick on the same GPU.  Weights N(0, 0.02), input N(0, 1) * 0.5,
    upstream gradient N(0, 1e-2); memory-efficient weight mode, first micro-batch (weight scales recomputed); gradients
    are reset to None before every step in both legs (no accumulation adds)."""
    import torch.nn.functional as F
    from coat_b200.activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
    from coat_b200.models.coat_llama import CoatLlamaConfig, CoatLlamaDecoderLayer
    from coat_b200.utils._fp8_quantization_config import QuantizationConfig
    from coat_b200.utils._fp8manager import FP8Manager
    Hd, I, heads, B, S = 4096, 11008, 32, 4, 2048
    qa = dict(group_size=16, weight_memory_efficient=True)
    cfg = CoatLlamaConfig(hidden_size=Hd, intermediate_size=I, num_attention_heads=heads, coat_fp8_args=qa)
    torch.manual_seed(3)
    layer = CoatLlamaDecoderLayer(cfg, 0)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0.0, 0.02) if p.dim() == 2 else p.fill_(1.0)
    layer = layer.to(device, torch.bfloat16).train()
    qargs = QuantizationConfig(**qa)
    bgn, end = Coat_quantize_bgn(qargs).train(), Coat_quantize_end(qargs).train()
    x = (torch.randn(B, S, Hd, device=device) * 0.5).to(torch.bfloat16).requires_grad_(True)
    up = (torch.randn(B, S, Hd, device=device) * 1e-2).to(torch.bfloat16)
    FP8Manager.is_first_microbatch = True

    def fp8_step():
        for p in layer.parameters():   # zero_grad(set_to_none=True), as a training step does: autograd then stores each
            p.grad = None              # gradient instead of adding it to last step's (a host-side reset, no kernel)
        x.grad = None
        (h, qh, sh), = layer(*bgn(x))
        end(h, qh, sh).backward(up)

    w = {n: p.detach().clone().requires_grad_(True) for n, p in layer.named_parameters()}

    def rms(t, g):
        return F.rms_norm(t, g.shape, g, 1e-5)

    def bf16_step():
        h = rms(x, w["input_layernorm.weight"])
        q, k, v = (F.linear(h, w[f"BeforeAttention.{n}_proj.weight"]).view(B, S, heads, Hd // heads).transpose(1, 2)
                   for n in "qkv")
        cos, sin = rope
        rot = lambda t: torch.cat((-t[..., t.shape[-1] // 2:], t[..., :t.shape[-1] // 2]), dim=-1)
        q, k = q * cos + rot(q) * sin, k * cos + rot(k) * sin
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, S, Hd)
        y = x + F.linear(a, w["AfterAttention.o_proj.weight"])
        h = rms(y, w["post_attention_layernorm.weight"])
        y = y + F.linear(F.silu(F.linear(h, w["MLPResidual.gate_proj.weight"])) *
                         F.linear(h, w["MLPResidual.up_proj.weight"]), w["MLPResidual.down_proj.weight"])
        for t in w.values():
            t.grad = None
        x.grad = None
        y.backward(up)

    from coat_b200.models.coat_llama import llama_rotary_embeddings
    pos = torch.arange(S, device=device)[None, :]
    rope = tuple(t.unsqueeze(1) for t in llama_rotary_embeddings(pos, Hd // heads, 10000.0, torch.bfloat16))
    out = {"tokens": B * S}

    def time_leg(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / iters

    if with_reference_operators:
        # the SAME composition on the reference's own operators (its Triton kernels with their own autotuning), as a
        # baseline on this GPU: the reference's functions are put in place of this package's in the layer module, the
        # weight cache and the quantise-in/out modules (oracle/ref_loader.py says which three calls are composed of
        # reference calls and which one operator, the RMSNorm backward, stays this package's on both sides)
        from oracle import ref_loader
        ref = ref_loader.load_ref_triton(one_config=False)
        if ref is None:
            out["fp8_layer_on_reference_operators"] = {"reference": "oracle/_ref/coat_ref not staged"}
        else:
            import coat_b200.activation.real_quantization as mine
            import coat_b200.activation.real_quantization.func_quantize as fq
            import coat_b200.models.coat_llama as layer_mod
            import coat_b200.utils._fp8_weightcache as cache_mod
            ops = ref_loader.reference_layer_operators(ref, mine)
            saved = []
            for mod in (layer_mod, cache_mod, fq):
                for name, fn in ops.items():
                    if hasattr(mod, name):
                        saved.append((mod, name, getattr(mod, name)))
                        setattr(mod, name, fn)
            try:
                ms = time_leg(fp8_step)
                out["fp8_layer_on_reference_operators"] = {"fwd_bwd_ms": ms, "tokens_per_s": B * S / (ms / 1e3)}
            except Exception as exc:
                out["fp8_layer_on_reference_operators"] = {"reference": f"did not run: {str(exc)[:160]}"}
            finally:
                for mod, name, fn in saved:
                    setattr(mod, name, fn)
    for name, fn in (("fp8_layer", fp8_step), ("bf16_torch_layer", bf16_step)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / iters
        out[name] = {"fwd_bwd_ms": ms, "tokens_per_s": B * S / (ms / 1e3)}
    out["fp8_over_bf16"] = out["bf16_torch_layer"]["fwd_bwd_ms"] / out["fp8_layer"]["fwd_bwd_ms"]
    ref_leg = out.get("fp8_layer_on_reference_operators", {})
    if "fwd_bwd_ms" in ref_leg:
        out["ours_over_reference_operators"] = ref_leg["fwd_bwd_ms"] / out["fp8_layer"]["fwd_bwd_ms"]
    return out


def olmo_block_extras(torch, device, iters=5, with_reference_operators=False):
    """Forward + backward of ONE OLMo-7B block (d_model 4096, 32 heads, ff_proj 22016, LayerNorm without parameters,
    SwiGLU) on 8 x 2048 tokens, the shape of the reference's per-layer benchmark (benchmark/benchmark_olmolayer.py):
    the FP8 block of this package, the same block in plain bf16 torch (cuBLAS GEMMs, SDPA, eager elementwise ops) and,
    on request, the same composition on the reference's own operators.  Weights by the block's own initialisation,
    input uniform in [0, 1) and upstream gradient uniform in [0, 1) as in that benchmark; memory-efficient weight mode,
    first micro-batch; gradients reset to None before every step in every leg."""
    import torch.nn.functional as F
    from coat_b200.activation.real_quantization.func_quantize import Coat_quantize_bgn, Coat_quantize_end
    from coat_b200.models.coat_olmo import CoatOLMoConfig, CoatOLMoSequentialBlock, olmo_rotary_tables
    from coat_b200.utils._fp8_quantization_config import QuantizationConfig
    from coat_b200.utils._fp8manager import FP8Manager
    D, HID, heads, B, T = 4096, 22016, 32, 8, 2048
    qargs = QuantizationConfig(group_size=16, weight_memory_efficient=True)
    cfg = CoatOLMoConfig(d_model=D, n_heads=heads, mlp_hidden_size=HID, max_sequence_length=T)
    torch.manual_seed(4)
    block = CoatOLMoSequentialBlock(0, cfg, qargs)
    block.reset_parameters()
    block = block.to(device, torch.bfloat16).train()
    bgn, end = Coat_quantize_bgn(qargs).train(), Coat_quantize_end(qargs).train()
    x = torch.rand(B, T, D, device=device).to(torch.bfloat16).requires_grad_(True)
    up = torch.rand(B, T, D, device=device).to(torch.bfloat16)
    FP8Manager.is_first_microbatch = True

    def fp8_step():
        for p in block.parameters():
            p.grad = None
        x.grad = None
        h, qh, sh, _ = block(*bgn(x))
        end(h, qh, sh).backward(up)

    w = {n: p.detach().clone().requires_grad_(True) for n, p in block.named_parameters()}
    sin, cos = (t.to(torch.bfloat16).unsqueeze(1) for t in olmo_rotary_tables(T, D // heads, 10000.0, device))

    def bf16_step():
        ln = lambda t: F.layer_norm(t, (D,), None, None, 1e-5)
        q, k, v = (t.view(B, T, heads, D // heads).transpose(1, 2)
                   for t in F.linear(ln(x), w["BeforeAttention.att_proj.weight"]).split((D, D, D), dim=-1))
        rot = lambda t: torch.cat((-t[..., t.shape[-1] // 2:], t[..., :t.shape[-1] // 2]), dim=-1)
        q, k = q * cos + rot(q) * sin, k * cos + rot(k) * sin
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, D)
        y = x + F.linear(a, w["AfterAttention.attn_out.weight"])
        u, g = F.linear(ln(y), w["MLPResidual.ff_proj.weight"]).chunk(2, dim=-1)
        y = y + F.linear(F.silu(g) * u, w["MLPResidual.ff_out.weight"])
        for t in w.values():
            t.grad = None
        x.grad = None
        y.backward(up)

    def time_leg(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / iters
        return {"fwd_bwd_ms": ms, "tokens_per_s": B * T / (ms / 1e3)}

    out = {"tokens": B * T}
    if with_reference_operators:
        from oracle import ref_loader
        ref = ref_loader.load_ref_triton(one_config=False)
        if ref is None:
            out["fp8_block_on_reference_operators"] = {"reference": "oracle/_ref/coat_ref not staged"}
        else:
            import coat_b200.activation.real_quantization as mine
            import coat_b200.activation.real_quantization.func_quantize as fq
            import coat_b200.models.coat_llama as llama_mod
            import coat_b200.models.coat_olmo as olmo_mod
            import coat_b200.utils._fp8_weightcache as cache_mod
            ops = ref_loader.reference_layer_operators(ref, mine)
            saved = []
            for mod in (olmo_mod, llama_mod, cache_mod, fq):
                for name, fn in ops.items():
                    if hasattr(mod, name):
                        saved.append((mod, name, getattr(mod, name)))
                        setattr(mod, name, fn)
            try:
                out["fp8_block_on_reference_operators"] = time_leg(fp8_step)
            except Exception as exc:
                out["fp8_block_on_reference_operators"] = {"reference": f"did not run: {str(exc)[:160]}"}
            finally:
                for mod, name, fn in saved:
                    setattr(mod, name, fn)
    out["fp8_block"] = time_leg(fp8_step)
    out["bf16_torch_block"] = time_leg(bf16_step)
    out["fp8_over_bf16"] = out["bf16_torch_block"]["fwd_bwd_ms"] / out["fp8_block"]["fwd_bwd_ms"]
    ref_leg = out.get("fp8_block_on_reference_operators", {})
    if "fwd_bwd_ms" in ref_leg:
        out["ours_over_reference_operators"] = ref_leg["fwd_bwd_ms"] / out["fp8_block"]["fwd_bwd_ms"]
    return out


def fused_extras(torch, device, peak):
    """GB/s of the fused quantize-on-save operators, the norms and the optimizer step without expansion, through the
    python operator API (the calls the decoder layer makes, with its arguments), on the benchmark shapes:
    8192 tokens x 11008 for the MLP operators, x 4096 for the residual adds and the norms; 4096 x 4096 fp32 for the
    optimizer.  Device time of 10 calls replayed from one CUDA graph (two input sets rotate; every operator moves
    more than L2 holds), median of 7 replays after a quarter of a second of warm-up replays.  Algorithmic bytes = compulsory reads + writes of the operator's
    inputs and outputs (FP8 codes 1 B, 1x16 bf16 scales 0.125 B/elem, bf16 2 B); the implementations move more
    where the reference's data flow forces a bf16 intermediate before a per-tensor scale is known."""
    import coat_b200.activation.real_quantization as r
    from coat_b200.optimizer import qoptim_cuda
    T, I, H = 8192, 11008, 4096
    gen = torch.Generator(device=device).manual_seed(4)

    def q16(M, N, scale=1.0):
        x = (torch.randn(M, N, generator=gen, device=device) * scale).to(torch.bfloat16)
        return r.fp8_quantize(x, 16, "E4M3")

    def bf(M, N, scale=1.0):
        return (torch.randn(M, N, generator=gen, device=device) * scale).to(torch.bfloat16)

    sets = []
    for _ in range(2):
        d = {"gate": q16(T, I), "up": q16(T, I), "g_i": bf(T, I, 1e-2), "h": q16(T, H), "a": bf(T, H), "b": bf(T, H),
             "g_h": bf(T, H, 1e-2)}
        d["w"] = (1 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.bfloat16)
        _, _, _, ctx = r.fp8_rmsnorm_forward(*d["h"], d["w"], 16, 1e-5)
        d["rstd"] = ctx[1]
        _, _, _, (d["mean"], d["ln_rstd"], _) = r.fp8_layernorm_noparam_forward(*d["h"], 16, 1e-5)
        sets.append(d)
    cases = {
        # name: (call on one input set, elements, algorithmic bytes per element)
        "silu_forward": (lambda d: r.fp8_silu_forward(*d["gate"], 16), T * I, 2.25),
        "mul_forward_pertensor_transposed": (lambda d: r.fp8_mul_forward(*d["gate"], *d["up"], 16, transpose_output_2d=True), T * I, 4.25),
        "mul_backward_pertensor_transposed": (lambda d: r.fp8_mul_backward(*d["gate"], *d["up"], d["g_i"], 16, "E5M2", output_quantized_transpose=True), T * I, 8.25),
        "silu_backward_pertensor_transposed": (lambda d: r.fp8_silu_backward(*d["gate"], d["g_i"], 16, "E5M2", output_quantized_transpose=True), T * I, 5.125),
        "silu_mul_forward_one_kernel": (lambda d: r.fp8_silu_mul_forward(*d["gate"], *d["up"], 16, transpose_output_2d=True), T * I, 5.375),
        "mul_silu_backward_one_kernel": (lambda d: r.fp8_mul_silu_backward(*d["gate"], *d["up"], *d["gate"], d["g_i"], 16, "E5M2"), T * I, 9.375),
        "gelu_forward_pertensor_transposed": (lambda d: r.fp8_gelu_forward(*d["gate"], 16, transpose_output_2d=True), T * I, 3.125),
        "add_fwd_bf16_and_1x16": (lambda d: r.fp8_add_Ifp_Ifp_Ofp_Og16(d["a"], d["b"], torch.float8_e4m3fn, 16), T * H, 7.125),
        "add_bwd_bf16_and_pertensor": (lambda d: r.fp8_add_Ifp_Ifp_Ofp_Opt(d["a"], d["g_h"], 16, "E5M2"), T * H, 7.125),
        "rmsnorm_forward_pertensor_transposed": (lambda d: r.fp8_rmsnorm_forward(*d["h"], d["w"], 16, 1e-5, transpose_output_2d=True), T * H, 3.125),
        "rmsnorm_backward": (lambda d: r.fp8_rmsnorm_backward(*d["h"], d["g_h"], d["w"], d["rstd"], 16, 8), T * H, 5.125),
        "layernorm_noparam_forward_pertensor_transposed": (lambda d: r.fp8_layernorm_noparam_forward(*d["h"], 16, 1e-5, transpose_output_2d=True), T * H, 3.125),
        "layernorm_noparam_backward": (lambda d: r.fp8_layernorm_noparam_backward(*d["h"], d["g_h"], 16, d["mean"], d["ln_rstd"], 8), T * H, 5.125),
    }
    # the optimizer step WITHOUT expansion (fp8_adamw_cuda_kernel.cu:21-125): 16.125 B per parameter
    n = 4096 * 4096
    opt_sets = []
    for _ in range(4):
        o = {"p": torch.randn(n, generator=gen, device=device) * 0.02, "g": torch.randn(n, generator=gen, device=device) * 1e-3,
             "m": torch.zeros(n, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
             "v": torch.zeros(n, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
             "s_m": torch.zeros(n // 128, device=device), "s_v": torch.zeros(n // 128, device=device)}
        qoptim_cuda.fp8_adamw_step(o["p"], o["g"], o["m"], o["s_m"], o["v"], o["s_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 128)
        opt_sets.append(o)
    step_no = [2]

    def plain_step(o):
        qoptim_cuda.fp8_adamw_step(o["p"], o["g"], o["m"], o["s_m"], o["v"], o["s_v"], 0.9, 0.95, 1e-4, 0.1, 1e-8,
                                   step_no[0], 128)

    out = {}
    iters = 10
    for name, (fn, elems, bpe) in list(cases.items()) + [("fp8_adamw_step_no_expansion", (plain_step, n, 16.125))]:
        data = opt_sets if fn is plain_step else sets
        for d in data:
            fn(d)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(iters):
                fn(data[i % len(data)])
        t_warm = time.time()
        while time.time() - t_warm < 0.25:   # warm-up until the clocks have ramped up (a cold process reads 2-3x slow)
            graph.replay()
            torch.cuda.synchronize(device)
        times = []
        for _ in range(7):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize(device)
            times.append(e0.elapsed_time(e1) / iters)
        del graph
        ms = sorted(times)[len(times) // 2]
        gbs = elems * bpe / (ms / 1e3) / 1e9
        out[name] = {"us": ms * 1e3, "GB/s": gbs, "frac_of_measured_hbm": gbs / peak, "algorithmic_bytes_per_elem": bpe}
        if fn is plain_step:
            out[name]["params_per_s"] = n / (ms / 1e3)
    return out


def fp8_peak_yardstick(torch, device):
    """A measured dense FP8 rate to quote the GEMM against: torch._scaled_mm (cuBLASLt) E4M3 x E4M3 -> bf16 at
    8192^3, best of 10 single launches (burst) and 300 launches back to back (sustained, power-capped).  A library
    GEMM used as a yardstick only; nothing in the product calls it."""
    n = 8192
    a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()   # column-major, as _scaled_mm wants
    one = torch.tensor(1.0, device=device)
    try:
        def call():
            return torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        for _ in range(3):
            call()
        torch.cuda.synchronize(device)
        best = 1e9
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            torch.cuda.synchronize(device)
            best = min(best, e0.elapsed_time(e1))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(300):
            call()
        e1.record()
        torch.cuda.synchronize(device)
        sustained = e0.elapsed_time(e1) / 300
    except Exception as exc:   # an image without an FP8 library GEMM: fall back to 2x the measured bf16 figures
        return {"unavailable": str(exc)[:160]}
    flop = 2.0 * n ** 3
    return {"how": "torch._scaled_mm e4m3 x e4m3 -> bf16, 8192^3", "burst_tflops": flop / (best / 1e3) / 1e12,
            "sustained_tflops": flop / (sustained / 1e3) / 1e12}


def reference_on_this_gpu(torch, device, peak):
    """The REFERENCE's own GPU kernels timed on this GPU beside this repository's, same inputs, same harness (python
    wrappers called back to back, CUDA events, median of 5 rounds of 20 calls after warm-up, which also lets the
    reference's autotuner settle): its compiled optimizer extension on the 4096 x 4096 tensor, its Triton quantizers
    on the 8192 x 4096 activation and its Triton FP8 matmul on the Llama-2-7B MLP shapes.  Baseline figures only:
    taken from the copies staged under oracle/_ref/ (absent -> the entry says so)."""
    from oracle import ref_loader
    import coat_b200.activation.real_quantization as mine
    from coat_b200.optimizer import qoptim_cuda as my_opt
    out = {}

    def timed(fn, rounds=5, calls=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        times = []
        for _ in range(rounds):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(calls):
                fn()
            e1.record()
            torch.cuda.synchronize(device)
            times.append(e0.elapsed_time(e1) / calls)
        return sorted(times)[len(times) // 2] * 1e3   # us

    def pair(name, ref_fn, my_fn, unit_work, unit):
        try:
            ref_us = timed(ref_fn)
        except Exception as exc:
            out[name] = {"reference": f"did not run: {str(exc)[:120]}"}
            return
        my_us = timed(my_fn)
        out[name] = {"reference_us": ref_us, "ours_us": my_us, "speedup": ref_us / my_us,
                     f"reference_{unit}": unit_work / ref_us, f"ours_{unit}": unit_work / my_us}

    ref_opt = ref_loader.load_ref_qoptim()
    if ref_opt is None:
        out["fp8_adamw_expand_4096x4096"] = {"reference": "oracle/_ref/qoptim_cuda.so not built"}
    else:
        n = 4096 * 4096
        gen = torch.Generator(device=device).manual_seed(0)

        def state():
            return dict(p=torch.randn(n, generator=gen, device=device) * 0.02,
                        g=torch.randn(n, generator=gen, device=device) * 1e-3,
                        m=torch.zeros(n, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
                        v=torch.zeros(n, dtype=torch.uint8, device=device).view(torch.float8_e4m3fn),
                        vec=[torch.zeros(n // 128, device=device), torch.ones(n // 128, device=device),
                             torch.ones(n // 128, device=device), torch.zeros(n // 128, device=device),
                             torch.ones(n // 128, device=device), torch.ones(n // 128, device=device)])
        sa, sb = state(), state()
        step = [1]

        def run(mod, st):
            s_m, k_m, r_m, s_v, k_v, r_v = st["vec"]
            step[0] += 1
            mod.fp8_adamw_expand_step(st["p"], st["g"], st["m"], s_m, k_m, r_m, st["v"], s_v, k_v, r_v, 0.9, 0.95, 1e-4,
                                      0.1, 1e-8, step[0], 128, 16)
        pair("fp8_adamw_expand_4096x4096", lambda: run(ref_opt, sa), lambda: run(my_opt, sb), n / 1e3, "Gparams_per_s")

    ref = ref_loader.load_ref_triton(one_config=False)
    if ref is None:
        out["triton_operators"] = {"reference": "oracle/_ref/coat_ref not staged"}
        return out
    M, N = 8192, 4096
    gen = torch.Generator(device=device).manual_seed(1)
    x = torch.randn(M, N, generator=gen, device=device)
    x = torch.where(torch.rand(M, N, generator=gen, device=device) < 1e-3, x * 100, x).to(torch.bfloat16)
    qt = ref_loader.ref_module("_quantize_transpose", one_config=False)
    gb = lambda bytes_per_elem: M * N * bytes_per_elem / 1e3   # -> GB/s when divided by us
    pair("fp8_quantize_1x16", lambda: ref.fp8_quantize(x, 16, "E4M3"), lambda: mine.fp8_quantize(x, 16, "E4M3"),
         gb(3.125), "GBps")
    pair("fp8_quantize_pertensor", lambda: ref.fp8_quantize_pertensor(x, 16, "E4M3"),
         lambda: mine.fp8_quantize_pertensor(x, 16, "E4M3"), gb(3.125), "GBps")
    pair("fp8_quantize_pertensor_transpose", lambda: ref.fp8_quantize_pertensor_transpose(x, 16, "E4M3"),
         lambda: mine.fp8_quantize_pertensor_transpose(x, 16, "E4M3"), gb(4.0), "GBps")
    pair("fp8_quantize_transpose_1x16", lambda: qt.fp8_quantize_transpose(x, 16, "E4M3"),
         lambda: mine.fp8_quantize_transpose(x, 16, "E4M3"), gb(4.25), "GBps")
    T, H, I = 8192, 4096, 11008
    gen = torch.Generator(device=device).manual_seed(2)
    X = torch.randn(T, H, generator=gen, device=device).to(torch.bfloat16)
    W = (torch.randn(I, H, generator=gen, device=device) * 0.02).to(torch.bfloat16)
    G = (torch.randn(T, I, generator=gen, device=device) * 1e-2).to(torch.bfloat16)
    qx, sx, qx_t = mine.fp8_quantize_pertensor_transpose(X, 16, "E4M3")
    qw, sw, qw_t = mine.fp8_quantize_pertensor_transpose(W, 16, "E4M3")
    qg, sg, qg_t = mine.fp8_quantize_pertensor_transpose(G, 16, "E5M2")
    tflop = 2.0 * T * H * I / 1e6   # -> TFLOP/s when divided by us
    pair("fp8_linear_forward_8192x11008x4096", lambda: ref.fp8_linear_forward(qx, sx, qw, sw, False, 16),
         lambda: mine.fp8_linear_forward(qx, sx, qw, sw, False, 16), tflop, "TFLOPs")
    pair("fp8_linear_backward_dgrad_and_wgrad",
         lambda: ref.fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, 16),
         lambda: mine.fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, 16), 2 * tflop, "TFLOPs")
    # the loss head: 4096 rows of fp32 logits over a 32000-entry vocabulary, loss and in-place gradient (the logits
    # are read once and overwritten once: 8 bytes per logit; what a call overwrites is the next call's input, softmax
    # gradients are as good a set of logits as any)
    liger = ref_loader.load_ref_liger()
    if liger is None:
        out["cross_entropy_4096x32000"] = {"reference": "oracle/_ref/coat_ref/activation/liger not staged"}
    else:
        from coat_b200.activation.liger import cross_entropy as my_ce
        rows, V = 4096, 32000
        gen = torch.Generator(device=device).manual_seed(3)
        la = torch.randn(rows, V, generator=gen, device=device) * 3
        lb = la.clone()
        tgt = torch.randint(0, V, (rows,), generator=gen, device=device)
        pair("cross_entropy_4096x32000",
             lambda: liger.cross_entropy_forward(la, tgt, -100, 0.0, 0.0, "mean", None, False),
             lambda: my_ce.cross_entropy_forward(lb, tgt, -100, 0.0, 0.0, "mean", None, False),
             rows * V * 8 / 1e3, "GBps")
    return out


def run_kernel_workload(args):
    """`--workload quantizers|gemm`: only those kernels, for profiling captures and quick checks."""
    import torch
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    peak, kind = measured_peaks()
    if args.workload == "quantizers":
        extras = {"quantizers_8192x4096_bf16": quantizer_extras(torch, device, peak)}
    elif args.workload == "fused":
        extras = {"fused_operators_8192_tokens": fused_extras(torch, device, peak)}
    elif args.workload == "blockscaled":
        extras = {"deepseek_blockscaled_llama2_7b_mlp": blockscaled_extras(torch, device, peak)}
    elif args.workload == "layer":
        extras = {"decoder_layer_llama2_7b_4x2048": layer_extras(torch, device, iters=max(1, min(args.steps, 10))),
                  "olmo_7b_block_8x2048": olmo_block_extras(torch, device, iters=max(1, min(args.steps, 10)))}
    elif args.workload == "reference-gpu":
        extras = {"reference_on_this_gpu": reference_on_this_gpu(torch, device, peak),
                  "decoder_layer_llama2_7b_4x2048": layer_extras(torch, device, with_reference_operators=True),
                  "olmo_7b_block_8x2048": olmo_block_extras(torch, device, with_reference_operators=True),
                  "fp8_peak_yardstick": fp8_peak_yardstick(torch, device)}
    else:
        extras = {"fp8_gemm_llama2_7b_mlp": gemm_extras(torch, device, iters=max(1, args.steps))}
    print(json.dumps({"metric": "extras only", "config": {"workload": args.workload}, "extras": extras}), flush=True)


def verify_gathered(opt, torch, dist):
    """After a step at N > 1: does EVERY rank's gathered buffer hold EVERY rank's updated weights?  Each rank
    checksums bf16(own fp32 shard) per bucket (a position-weighted sum of the bit patterns, int64) and the matching
    slots of all ranks in its own gathered buffer; the own-shard checksums are all-gathered over NCCL and compared.
    Returns True only if all slots on all ranks agree."""
    dev = opt.device
    W, rank = opt.world_size, opt.rank

    def checksum(t_bf16):
        bits = t_bf16.contiguous().view(torch.int16).to(torch.int64)
        weight = (torch.arange(bits.numel(), device=dev, dtype=torch.int64) % 65521) + 1
        return (bits * weight).sum()

    own, seen = [], []
    for b in range(opt.n_buckets):
        lo, hi = int(opt.bounds[b]) * 128, int(opt.bounds[b + 1]) * 128
        own.append(checksum(opt.param[lo:hi].to(torch.bfloat16)))
        slots = opt._bucket_all[b].view(W, hi - lo)
        seen.append(torch.stack([checksum(slots[r]) for r in range(W)]))
    own = torch.stack(own)                         # [buckets]
    seen = torch.stack(seen)                       # [buckets, W]
    everyone = [torch.empty_like(own) for _ in range(W)]
    dist.all_gather(everyone, own)
    expected = torch.stack(everyone, dim=1)        # [buckets, W]
    ok = torch.tensor([int(torch.equal(seen, expected))], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return bool(ok.item())


def run_gpu_arm(args):
    import torch
    import torch.distributed as dist
    from coat_b200.sharded import ShardedCoatAdamW

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU path for the product)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        # the bucketed all-gather runs under the step kernels: give NCCL's stream priority over them
        opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        dist.init_process_group("nccl", device_id=device, pg_options=opts)

    shapes = llama2_7b_shapes() if args.workload == "llama2-7b" else [(4096, 4096)]
    numels = [numel(s) for s in shapes]
    total = sum(numels)
    exchange, exchange_note = (args.exchange if world > 1 else None), ""
    if exchange == "auto":
        exchange = "copy" if world == 2 else "p2p"   # ShardedCoatAdamW's own default, spelled out for the record
    try:
        opt = ShardedCoatAdamW(numels, rank=rank, world_size=world, device=device, exchange=exchange,
                               copy_peers=args.copy_peers, n_buckets=args.buckets, **HYPER)
    except RuntimeError as e:   # raised on every rank alike when the peer mapping is not available
        if exchange not in ("p2p", "copy", "hybrid"):
            raise
        exchange, exchange_note = "nccl", f" ({exchange} set-up failed: {str(e)[:200]})"
        opt = ShardedCoatAdamW(numels, rank=rank, world_size=world, device=device, exchange="nccl", **HYPER)
    fill_synthetic(opt, shapes, torch)
    my_params = sum(pc.numel for pc in opt.my_pieces)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # two independent gradient sets, alternated, so that the moments do not converge onto one
    # fixed gradient (a single repeated gradient makes the requantisation unrealistically easy)
    grads = [opt.grad, torch.empty_like(opt.grad).normal_(0.0, 1e-3)]
    for gbuf in grads:   # device-side tensor tables of both gradient sets are built outside the timed region
        opt.set_grad_buffer(gbuf)
    step_no = [0]

    def one_step(local_only=False):
        opt.set_grad_buffer(grads[step_no[0] & 1])
        step_no[0] += 1
        opt.local_step() if local_only else opt.step()

    for _ in range(max(args.warmup, 3)):
        one_step()
    barrier()
    sampler = ClockSampler(local)
    if rank == 0:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(args.steps):
        one_step()
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps

    # the fused kernel alone (no collective), for the roofline
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for _ in range(args.steps):
        one_step(local_only=True)
    k1.record()
    torch.cuda.synchronize(device)
    kernel_ms = k0.elapsed_time(k1) / args.steps
    clocks = sampler.stop() if rank == 0 else None

    t = torch.tensor([ms, kernel_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kernel_ms = t.tolist()
    n_launches = args.steps * opt.n_buckets
    gather_verified = None
    if world > 1:   # one more full step (the kernel-only steps above exchanged nothing), then compare the buffers
        one_step()
        barrier()
        gather_verified = verify_gathered(opt, torch, dist)
    opt.close()   # collective: unmaps the peers' buffers

    # end to end through the public API with host buffers: every rank steps its own copy of one decoder layer
    # over its own PCIe link at the same time; the job's rate is all ranks' parameters over the slowest rank's time
    e2e_v, h2d, d2h, e2e_n = None, 0, 0, 0
    if not args.kernel_only:
        e2e_ms, h2d, d2h, e2e_n = e2e_public_api(torch, device, max(3, min(args.steps, 10)), args.warmup)
        t2 = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e_v = world * e2e_n / (t2.item() / 1e3)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = my_params * BYTES_PER_PARAM_BF16 / (kernel_ms / 1e3) / 1e9
        # measured DRAM bytes per parameter (see the constants above) times this launch's parameter count: the
        # full-size figure for launches that stream far more than L2 holds, the small case's for the small case
        per_param = NCU_DRAM_BYTES_PER_PARAM_FULL if my_params * BYTES_PER_PARAM_BF16 > 4e9 else NCU_DRAM_BYTES_PER_PARAM_C1
        traffic = per_param * my_params
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": traffic, "peak_kind": f"of {peak_kind}", "kernel": "fp8_adamw_expand_tiled_kernel<float,table>",
                    "kernel_ms": kernel_ms, "algorithmic_bytes_per_param": BYTES_PER_PARAM_BF16}
        if args.kernel_only or world > 1:  # profiling runs: nothing but the fused kernel; the CPU leg runs at N = 1
            cpu_v = cpu_steps = cpu_dt = cores = None
        else:
            cpu_v, cpu_steps, cpu_dt, cores = cpu_reference_steps(4096 * 4096, 10.0)
        line = {
            "metric": METRIC, "value": total / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 math / e4m3 state", "data": "synthetic",
            "config": workload_config(world, exchange, args.workload, exchange_note),
            # the step alone (no exchange) and what the exchange adds, so that the scaling of the two can be told apart
            "step_only": {"value": total / (kernel_ms / 1e3), "unit": UNIT, "ms_per_step": kernel_ms},
            "exchange": None if world == 1 else {
                "kind": exchange, "ms_beyond_step": ms - kernel_ms,
                "bf16_bytes_received_per_gpu": 2 * opt.plan.shard_numel * (world - 1),
                "link_bound_ms": 2 * opt.plan.shard_numel * (world - 1) / 770e9 * 1e3,
                "link_rate_note": "770 GB/s per direction per GPU: the peer-copy rate measured on this pool",
                "gather_verified": gather_verified},
            "roofline": roofline,
            "e2e": {"value": e2e_v, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "workload": f"CoatAdamW.step on one decoder layer ({e2e_n} params) per GPU, grads from pinned "
                                "host memory, updated fp32 weights read back; bytes are per GPU"},
            "gpu_launches": n_launches,
            "clocks": clocks,
        }
        if not args.kernel_only and args.workload == "llama2-7b" and world == 1:
            del opt, grads
            torch.cuda.empty_cache()
            line["extras"] = {"quantizers_8192x4096_bf16": quantizer_extras(torch, device, peak),
                              "fused_operators_8192_tokens": fused_extras(torch, device, peak),
                              "fp8_gemm_llama2_7b_mlp": gemm_extras(torch, device),
                              "decoder_layer_llama2_7b_4x2048": layer_extras(torch, device, with_reference_operators=True),
                              "olmo_7b_block_8x2048": olmo_block_extras(torch, device, with_reference_operators=True),
                              "deepseek_blockscaled_llama2_7b_mlp": blockscaled_extras(torch, device, peak),
                              "reference_on_this_gpu": reference_on_this_gpu(torch, device, peak)}
        if cpu_v is not None:
            line["cpu_baseline"] = {
                "value": cpu_v, "unit": UNIT, "cores": cores, "kind": "port",
                "sample": f"{cpu_steps} steps of one 4096x4096 tensor in {cpu_dt:.1f} s, C restatement of the "
                          f"reference kernel with OpenMP over groups, {cores} threads",
                "pure_pytorch": cpu_pure_pytorch_steps()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama2-7b", choices=["llama2-7b", "c1", "quantizers", "fused", "gemm", "layer", "blockscaled", "reference-gpu"],
                    help="c1 = one 4096x4096 tensor, the small case used for ncu captures")
    ap.add_argument("--buckets", type=int, default=None,
                    help="bucketed exchanges: number of buckets the shard is cut into (default: 8)")
    ap.add_argument("--copy-peers", type=int, default=None,
                    help="hybrid exchange: how many peers the DMA engines serve (default: about a third)")
    ap.add_argument("--exchange", default="auto", choices=["auto", "p2p", "nccl", "copy", "hybrid"],
                    help="how the bf16 weights reach the other ranks at --gpus > 1: stored into the peers' buffers by "
                         "the step kernel itself, or bucketed NCCL all-gathers overlapped with the step")
    ap.add_argument("--kernel-only", action="store_true", help="skip the e2e and CPU legs (profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
    elif args.workload in ("quantizers", "fused", "gemm", "layer", "blockscaled", "reference-gpu"):
        run_kernel_workload(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
