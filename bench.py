"""Benchmark of the B200 KDA layer (forward + backward), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg1|cfg2|cfg3|cfg4|decode]

Step = one forward + backward of the KDA layer (ShortConv+SiLU, L2 norms,
gate, beta, chunked gated delta rule) over one batch of synthetic inputs of
configuration 1 (8 sequences x 4096 tokens x 16 heads x 128, bf16, fp32 state)
per GPU, then one NCCL all-reduce of the layer's weight gradients when N > 1
(weak scaling: every rank processes its own 8 sequences).  The all-reduce is
asynchronous: it runs on NCCL's stream while the next step computes, and the
timed region ends after the last one completes.  ``--workload cfg3`` is one
optimizer update of configuration 3: its 320 sequences sharded over the ranks
(strong scaling), each rank running its share as micro-batches of at most
40 sequences with the weight gradients accumulated, then one all-reduce (320
sequences fwd+bwd need about 181 GB of activations, saved products and
workspace at once, more than one GPU holds);
``--workload cfg2`` steps the whole mixer block of configuration 2
(``sophia_b200.mixer.KDAMixerBlock``: input RMSNorm, fused q/k/v/gate GEMM,
decay and beta projections, the KDA layer, gated output RMSNorm, out-
projection; 4 x 4096 tokens, hidden 1536, bf16 autocast) per GPU;
``--workload cfg4`` steps configuration 4's packed ragged batch per GPU: 16
windows of 4096 tokens holding documents of log-uniform length in [32, 4096]
(seed 42), one 65,536-token sequence with ``cu_seqlens`` built on the device
from the windows' end-of-document tokens every step (``document_cu_seqlens``);
``--workload decode`` steps ``kda_decode`` calls of one token for each of 256
sequences (ShortConv with its history + the fp32 recurrence, state carried;
the line's roofline is the decode kernel's state traffic against HBM).

Timing: W untimed warm-up steps, then K steps between a barrier +
synchronize on both sides, CUDA events on the launch stream, max over ranks.
Inputs (q, k, v, g, dO: 128 MiB each) exceed the 126 MB L2, so no flush is
needed between steps.  The ``e2e`` figure repeats the step through the public
API with the step's inputs copied from pinned host memory and the weight
gradients read back each step (the input copies run on a second stream, so
step i+1's inputs cross PCIe while step i computes).  ``--impl reference`` times the reference's CPU
implementation (the oracle restatement of ``SophiaKDA._reference_kda`` +
``CausalDepthwiseConv1d`` with autograd) on the host cores instead.  Both CPU
figures (that arm, and the ``cpu_baseline`` of this one) time the same sample:
one sequence of ``CPU_SAMPLE_TOKENS`` tokens x 16 heads, fwd+bwd (the
reference's loop costs the same per token at any length, so the rate stands
for configuration 1's sequences).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "KDA layer fwd+bwd tokens/s at H=16,D=128,T=4096 (1/2/4/8 B200) + % roofline"
H, D, T = 16, 128, 4096
CFG3_SEQS, CFG3_MICRO = 320, 40  # configuration 3: sequences per update, sequences per micro-batch
CPU_SAMPLE_TOKENS = 1024         # tokens of the timed CPU sample (both CPU figures)

# Algorithmic HBM bytes per token-head of each kernel (reads + writes of its
# interface tensors, each once; bf16 activations, fp32 per-chunk vectors).
KERNEL_BYTES_PER_TOKEN_HEAD = {
    "fwd_intra": 1026 + 2700,   # q,k,v,g,beta in; W,U,Qt,Kbar,M,2^Gam_C, A and L' (bf16 64x64 per chunk)
                                # and the saved products q_hat,k_hat,v (bf16), Gam (fp32), beta out
    "fwd_state": 1160 + 1024,   # W,U,Qt,Kbar,M,2^Gam_C in; o, chunk states, v_new out
    "bwd_state": 1928 + 1160,   # W,Qt,Kbar,M,2^Gam_C,v_new,dO,chunk states in; dE,dQt,dW,dKbar,dM,dGam_C out
    "bwd_intra": 2956 + 1042,   # saved products, g, A, L' + dE,dW,dQt,dKbar,dM,dGam_C in;
                                # dq_hat,dk_hat,dv,dg,dbeta,partials out
    "bwd_post": 1536 + 768,     # q,k,v and dq_hat,dk_hat,dv in; dq,dk,dv out
}
# Tensor-core FLOPs per token-head of each kernel (algorithmic, no recompute).
KERNEL_FLOPS_PER_TOKEN_HEAD = {
    "fwd_intra": 2 * (2 * 64 * 128 + 2 * 64 * 128) + 2731,  # L', M, W, U and the inverse
    "fwd_state": 2 * 3 * 128 * 128 + 2 * 64 * 128,          # E, O (state part + M E), S update
    "bwd_state": 2 * 2 * (2 * 3 * 128 * 128 + 2 * 64 * 128),
    "bwd_intra": 2 * 2 * (2 * (2 * 64 * 128 + 2 * 64 * 128) + 2731),
    "bwd_post": 0,
}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per token-head of
# each kernel from one ncu capture of `python bench.py --batch 2 --steps 1
# --warmup 3 --profile` (B=2: the per-launch traffic scales with the token-heads
# processed).
NCU_DRAM_BYTES_PER_TOKEN_HEAD: dict[str, float] = {
    "fwd_intra": 3339.2, "fwd_state": 1872.2, "bwd_state": 2864.0, "bwd_intra": 3850.9, "bwd_post": 2226.1,
}
# The device code of the layer's kernels (the headers they are built from) and its
# hash when that capture ran: the line says whether the traffic figures describe
# the kernels being timed.
LAYER_KERNEL_SOURCES = ("kda_bwd_intra.cuh", "kda_bwd_state_tc.cuh", "kda_common.cuh", "kda_fwd.cuh",
                        "kda_fwd_state_tc.cuh", "kda_intra.cuh", "kda_post.cuh", "kda_tc.cuh")
NCU_SOURCE_HASH = "063c51444baa7a1d"


def kernel_source_hash() -> str:
    import hashlib
    h = hashlib.sha256()
    for f in LAYER_KERNEL_SOURCES:
        with open(os.path.join(ROOT, "sophia_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4", "decode"], default="cfg1")
    ap.add_argument("--profile", action="store_true",
                    help="run the warm-up and K layer steps only, print nothing (command for ncu captures)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per rank (default 8 for cfg1); smaller for ncu captures")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons sampled every 10 ms through NVML in a
    background thread; only samples taken inside the timed window (host time
    from the opening synchronize to the closing one) are kept."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device: torch.device):
        self.samples: list[tuple[float, float, int]] = []
        self.window = (0.0, 0.0)
        self.error = None
        self.stop_evt = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(device).uuid)
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report it instead of clocks
            self.nvml, self.error = None, f"nvml unavailable: {e}"

    def _poll(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_evt.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                self.samples.append((time.perf_counter(), float(mhz), int(get_reasons(self.handle))))
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(0.01)

    def start(self):
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self):
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error], "samples": 0}
        self.stop_evt.set()
        self.thread.join(timeout=2)
        t0, t1 = self.window
        inside = [(m, r) for t, m, r in self.samples if t0 <= t <= t1]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [self.error or "no samples"],
                    "samples": 0}
        reasons = set()
        for name, const in self.REASONS:
            bit = getattr(self.nvml, const, 0)
            if any(r & bit for _, r in inside):
                reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in inside), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(inside)}


CFG4_WINDOWS = 16
CFG4_EOS, CFG4_CAPACITY = 0, 128  # the end-of-document token; document-table capacity (95 documents)


def cfg4_cu_seqlens(windows: int = CFG4_WINDOWS, seed: int = 42) -> list[int]:
    """Configuration 4's packed document boundaries: each 4096-token window is
    filled with documents of log-uniform length in [32, 4096] (drawn with a
    generator seeded per window, the last cut at the window end); the windows
    are concatenated into one sequence of windows x 4096 tokens."""
    cu = [0]
    for w in range(windows):
        gen = torch.Generator().manual_seed(seed * 1000 + w)
        used = 0
        while used < T:
            u = torch.rand(1, generator=gen).item()
            n = min(int(round(math.exp(math.log(32) + u * (math.log(4096) - math.log(32))))), T - used)
            used += n
            cu.append(cu[-1] + n)
    return cu


def cfg4_tokens(device) -> torch.Tensor:
    """Configuration 4's token windows [windows, 4096] int32: random token ids
    with the end-of-document token at the last token of every document that ends
    inside a window (a window start begins a document anyway)."""
    gen = torch.Generator().manual_seed(4242)
    tok = torch.randint(1, 50000, (CFG4_WINDOWS * T,), generator=gen, dtype=torch.int32)
    for b in cfg4_cu_seqlens()[1:-1]:
        if b % T:
            tok[b - 1] = CFG4_EOS
    return tok.view(CFG4_WINDOWS, T).to(device)


def make_inputs(B, device, seed, Tlen=T):
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s, std=1.0: torch.randn(*s, device=device, generator=g) * std  # noqa: E731
    x = {k: rn(B, Tlen, H, D).to(torch.bfloat16) for k in ("q", "k", "v", "g")}
    x["beta"] = rn(B, Tlen, H).to(torch.bfloat16)
    x["do"] = rn(B, Tlen, H, D).to(torch.bfloat16)
    w = {"A_log": torch.zeros(H, device=device), "dt_bias": torch.zeros(H * D, device=device)}
    for k in ("conv_q", "conv_k", "conv_v"):
        w[k] = rn(H * D, 4, std=0.5)
    return x, w


def bench_ours(a, rank, world, local_rank):
    import torch.distributed as dist
    from sophia_b200 import _lib, document_cu_seqlens, dp, kda_layer

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # cfg1: 8 sequences per rank (weak scaling); cfg3: rank's share of 320 (strong)
    packed = a.workload == "cfg4"
    if packed:  # one sequence of 16 packed windows, documents reset at cu_seqlens
        B, Tlen = 1, CFG4_WINDOWS * T
        cu = None  # built on the device from the windows' tokens in every step
    else:
        B = a.batch or (8 if a.workload == "cfg1" else len(range(CFG3_SEQS)[dp.shard(CFG3_SEQS, rank, world)]))
        Tlen, cu = T, None
    # cfg3: the rank's B sequences run as micro-batches of at most CFG3_MICRO
    # (the same synthetic micro-batch each time), gradients accumulated
    micro = min(B, CFG3_MICRO) if a.workload == "cfg3" else B
    n_micro = -(-B // micro)
    x, w = make_inputs(micro, device, 42 + rank, Tlen)
    if packed:
        x["tok"] = cfg4_tokens(device)
    acts = {k: x[k].clone().requires_grad_(True) for k in ("q", "k", "v", "g", "beta")}
    params = {k: v.clone().requires_grad_(True) for k, v in w.items()}
    bucket = torch.empty(dp.bucket_numel(H, D), device=device, dtype=torch.float32)
    pending = []  # the in-flight all-reduce of the previous step

    def drain():
        while pending:
            pending.pop().wait()

    def step(inputs=None):
        """inputs: None (the resident micro-batch every time) or a function of
        the micro-batch index returning that micro-batch's inputs."""
        for t in list(params.values()):
            t.grad = None
        for mb in range(n_micro):
            src = acts if inputs is None else inputs(mb)
            rows = min(micro, B - mb * micro)
            for t in src.values():
                t.grad = None
            sl = (lambda t: t) if rows == micro else (lambda t: t[:rows])  # noqa: E731
            cu_mb = cu
            if packed:  # the data path's document table, capture-safe (no host sync)
                cu_mb, _ = document_cu_seqlens(x["tok"] if inputs is None else src["_tok"], CFG4_EOS,
                                               CFG4_CAPACITY)
            o, _ = kda_layer(sl(src["q"]), sl(src["k"]), sl(src["v"]), sl(src["g"]), sl(src["beta"]),
                             params["A_log"], params["dt_bias"], params["conv_q"], params["conv_k"],
                             params["conv_v"], cu_seqlens=cu_mb)
            o.backward(sl(x["do"] if inputs is None else src["_do"]))
        drain()  # the previous step's reduction reads the bucket
        dp.grad_bucket(params, out=bucket)
        h = dp.allreduce_bucket_async(bucket)
        if h is not None:
            pending.append(h)
        return bucket

    def timed(fn, steps, sampler=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        drain()
        e1.record(st)
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.mark(h0, time.perf_counter())
        if world > 1:
            dist.barrier()
        return dp.max_over_ranks(e0.elapsed_time(e1), device)

    for _ in range(a.warmup):
        step()
    if a.profile:
        timed(step, a.steps)
        return None
    sampler = ClockSampler(device)
    sampler.start()
    ms = timed(step, a.steps, sampler)
    clocks = sampler.stop()
    rank_tokens = B * Tlen
    global_tokens = CFG3_SEQS * T if a.workload == "cfg3" else world * rank_tokens
    tokens = global_tokens * a.steps
    value = tokens / (ms / 1e3)

    # per-kernel device times (second pass, CUDA events around every launch)
    _lib.timing_reset()
    _lib.timing_enable(True)
    ms_prof = timed(step, a.steps)
    _lib.timing_enable(False)
    kern = _lib.timing_read()
    _lib.timing_reset()
    launches = sum(n for n, _ in kern.values())

    # end to end through the public API: every micro-batch of every step
    # copies its inputs from pinned host memory, and every step reads the
    # weight gradients back.  The copies run on a second stream into two
    # alternating device buffers, so micro-batch i+1's inputs cross PCIe while
    # micro-batch i computes; all copies are inside the timed region.
    host = {k: x[k].cpu().pin_memory() for k in ("q", "k", "v", "g", "beta", "do") + (("tok",) if packed else ())}
    bufs = [{k: torch.empty_like(x[k]) for k in host} for _ in range(2)]
    out_host = torch.empty(bucket.numel(), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(device=device)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        copy_stream.wait_event(e0)

        def issue_copy(i):
            b = i % 2
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(freed[b])  # step i-2 is done with this buffer
                for k in host:
                    bufs[b][k].requires_grad_(False)
                    bufs[b][k].copy_(host[k], non_blocking=True)
                copied[b].record(copy_stream)

        total = steps * n_micro
        issue_copy(0)
        state = {"i": 0}

        def micro_inputs(_mb):
            i = state["i"]
            if i > 0:  # the previous micro-batch's buffer is free once its kernels ran
                freed[(i - 1) % 2].record(st)
            if i + 1 < total:
                issue_copy(i + 1)
            b = i % 2
            st.wait_event(copied[b])
            inp = {k: bufs[b][k].requires_grad_(True) for k in ("q", "k", "v", "g", "beta")}
            inp["_do"] = bufs[b]["do"]
            if packed:
                inp["_tok"] = bufs[b]["tok"]
            state["i"] = i + 1
            return inp

        for _ in range(steps):
            step(micro_inputs)
            drain()
            out_host.copy_(bucket, non_blocking=True)
        e1.record(st)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return dp.max_over_ranks(e0.elapsed_time(e1), device)

    e2e_run(2)
    e2e_steps = max(3, min(a.steps, 10))
    ms_e2e = e2e_run(e2e_steps)
    h2d = n_micro * sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    hbm, tc, tc_sus, src = peaks()
    # dominant kernel and its roofline
    th = micro * Tlen * H  # token-heads per launch
    dom = max((k for k in kern if k in KERNEL_BYTES_PER_TOKEN_HEAD), key=lambda k: kern[k][1])
    n_l, tot = kern[dom]
    per_launch_ms = tot / max(1, n_l)
    alg_bytes = KERNEL_BYTES_PER_TOKEN_HEAD[dom] * th
    achieved = alg_bytes / (per_launch_ms / 1e3) / 1e9
    traffic = None
    if dom in NCU_DRAM_BYTES_PER_TOKEN_HEAD:
        traffic = round(NCU_DRAM_BYTES_PER_TOKEN_HEAD[dom] * th)
    traffic_current = kernel_source_hash() == NCU_SOURCE_HASH
    # per-kernel roofline of the whole step: sum_k max(F_k/P, B_k/BW)
    roof_ms = 0.0
    for k, bpt in KERNEL_BYTES_PER_TOKEN_HEAD.items():
        f = KERNEL_FLOPS_PER_TOKEN_HEAD[k] * th
        roof_ms += max(f / (tc_sus * 1e12), bpt * th / (hbm * 1e9)) * 1e3
    roof_ms *= n_micro  # launches of each kernel per step
    kernel_ms_per_step = {k: round(v[1] / a.steps, 4) for k, v in kern.items() if v[0]}
    return {
        "value": value, "ms": ms / a.steps, "B": B, "micro": micro, "n_micro": n_micro, "clocks": clocks,
        "e2e": {"value": global_tokens * e2e_steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4), "traffic": traffic,
                     "traffic_source": "ncu dram bytes at B=2 scaled to this launch; current kernel sources: "
                                       + ("yes" if traffic_current else "no (stale)"),
                     "peak_source": src,
                     "per_kernel_roofline_ms": round(roof_ms, 4),
                     "per_kernel_roofline_frac": round(roof_ms / (ms_prof / a.steps), 4),
                     "kernel_ms_per_step": kernel_ms_per_step},
    }


def cpu_sample(tokens: int, threads: int | None = None):
    """The reference's CPU path (oracle restatement) fwd+bwd on one sequence
    of `tokens` tokens x 16 heads, fp32, torch autograd.  Returns tokens/s."""
    sys.path.insert(0, ROOT)
    from oracle.kda_oracle import kda_layer as oracle_layer
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    mk = lambda *s, std=1.0: (torch.randn(*s, generator=g) * std).requires_grad_(True)  # noqa: E731
    q, k, v, gg = (mk(1, tokens, H, D) for _ in range(4))
    beta = mk(1, tokens, H)
    A, dtb = torch.zeros(H, requires_grad=True), torch.zeros(H * D, requires_grad=True)
    convs = [mk(H * D, 4, std=0.5) for _ in range(3)]
    do = torch.randn(1, tokens, H, D, generator=g)
    t0 = time.perf_counter()
    out = oracle_layer(q, k, v, gg, beta, A, dtb, conv_weights=convs, compute_dtype=torch.float32)
    (out.o * do).sum().backward()
    dt = time.perf_counter() - t0
    return tokens / dt, dt


DECODE_METRIC = ("KDA decode tokens/s at B=256 sequences,H=16,D=128, one token per sequence per call "
                 "(fp32 state) + % roofline")
DECODE_BATCH = 256  # the fp32 states (268 MB) exceed L2, so every call streams them from HBM
# DRAM bytes per decode call and sequence, from one ncu capture of `python bench.py
# --workload decode --steps 20 --warmup 3` (dram__bytes_read.sum + dram__bytes_write.sum,
# kda_recurrent_kernel, B = 256: 291.7 MB read + 233.8 MB written per launch)
NCU_DECODE_DRAM_BYTES_PER_SEQ = 525.5e6 / 256


def decode_bytes_per_step(B: int) -> int:
    """Algorithmic HBM bytes of one decode call: the fp32 state read and written,
    the conv history read and written, the bf16 token inputs and output, the
    per-head weights."""
    state = B * H * D * D * 4 * 2
    conv = B * 3 * H * D * 3 * 4 * 2
    io = B * H * D * 2 * 5 + B * H * 2
    weights = H * D * 4 * (1 + 3 * 4) + H * 4
    return state + conv + io + weights


def cpu_decode_sample(B: int, steps: int, threads: int | None = None):
    """The reference's CPU decode (oracle restatement of the per-token
    recurrence, fp32, no gradients): `steps` calls of one token for B
    sequences x 16 heads, the state carried.  Returns tokens/s."""
    sys.path.insert(0, ROOT)
    from oracle.kda_oracle import kda_layer as oracle_layer
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    mk = lambda *s, std=1.0: torch.randn(*s, generator=g) * std  # noqa: E731
    A, dtb = torch.zeros(H), torch.zeros(H * D)
    state = mk(B, H, D, D, std=0.1)
    t0 = time.perf_counter()
    with torch.no_grad():
        for _ in range(steps):
            q, k, v, gg = (mk(B, 1, H, D) for _ in range(4))
            out = oracle_layer(q, k, v, gg, mk(B, 1, H), A, dtb, initial_state=state, compute_dtype=torch.float32)
            state = out.final_state
    dt = time.perf_counter() - t0
    return B * steps / dt, dt


def bench_decode(a, rank, world, local_rank):
    """Decode steps through ``sophia_b200.kda_decode`` (the cached-continuation
    path: ShortConv with its history + the fp32 recurrence, one fused kernel),
    one token per sequence per call, the state and the conv history carried
    from call to call (weak scaling over ranks: each rank decodes its own B
    sequences; inference, so no collective)."""
    import torch.distributed as dist
    from sophia_b200 import _lib, kda_decode

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    B = a.batch or DECODE_BATCH
    g = torch.Generator(device=device).manual_seed(42 + rank)
    rn = lambda *s, std=1.0: torch.randn(*s, device=device, generator=g) * std  # noqa: E731
    x = {k: rn(B, 1, H, D).to(torch.bfloat16) for k in ("q", "k", "v", "g")}
    x["beta"] = rn(B, 1, H).to(torch.bfloat16)
    A_log, dt_bias = torch.zeros(H, device=device), torch.zeros(H * D, device=device)
    taps = [rn(H * D, 4, std=0.5) for _ in range(3)]
    conv_state = rn(B, 3, H * D, 3)
    box = {"state": rn(B, H, D, D, std=0.1)}

    def step(src=None):
        src = x if src is None else src
        o, ht = kda_decode(src["q"], src["k"], src["v"], src["g"], src["beta"], A_log, dt_bias, *taps,
                           conv_state, initial_state=box["state"])
        box["state"] = ht
        return o

    def timed(fn, steps, sampler=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.mark(h0, time.perf_counter())
        if world > 1:
            dist.barrier()
        from sophia_b200 import dp
        return dp.max_over_ranks(e0.elapsed_time(e1), device)

    with torch.no_grad():
        for _ in range(max(a.warmup, 3)):
            step()
        sampler = ClockSampler(device)
        sampler.start()
        ms = timed(step, a.steps, sampler)
        clocks = sampler.stop()
        _lib.timing_reset()
        _lib.timing_enable(True)
        timed(step, a.steps)
        _lib.timing_enable(False)
        kern = _lib.timing_read()
        _lib.timing_reset()
        launches = sum(n for n, _ in kern.values())
        # end to end: each call's inputs copied from pinned host memory, its output read back
        host = {k: x[k].cpu().pin_memory() for k in ("q", "k", "v", "g", "beta")}
        dev = {k: torch.empty_like(x[k]) for k in host}
        out_host = torch.empty(B, 1, H, D, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            for k in host:
                dev[k].copy_(host[k], non_blocking=True)
            out_host.copy_(step(dev), non_blocking=True)

        ms_e2e = timed(e2e_step, a.steps)
    hbm, _, _, src = peaks()
    n_k, k_ms = kern.get("recurrent", (0, 0.0))
    per_launch = k_ms / max(1, n_k)
    alg = decode_bytes_per_step(B)
    achieved = alg / (per_launch / 1e3) / 1e9 if per_launch > 0 else 0.0
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    return {
        "value": world * B * a.steps / (ms / 1e3), "ms": ms / a.steps, "clocks": clocks,
        "e2e": {"value": world * B * a.steps / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": "recurrent", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "traffic": round(NCU_DECODE_DRAM_BYTES_PER_SEQ * B),
                     "traffic_source": "ncu dram bytes of this workload at B=256, scaled by the sequences",
                     "peak_source": src, "bytes_per_launch": alg, "kernel_ms_per_step": {k: round(v[1] / a.steps, 4)
                                                                     for k, v in kern.items() if v[0]}},
    }


MIXER_METRIC = "KDA mixer block fwd+bwd tokens/s at B=4,T=4096,hidden 1536,H=16,D=128 (cfg2) + % roofline"
DIM, DECAY_RANK = 1536, 128


def mixer_flops_per_token() -> float:
    """Algorithmic FLOPs per token of the block, fwd+bwd: its GEMMs (2 m n k
    per token, x3 for fwd+bwd) and the KDA layer's tensor FLOPs (16 heads)."""
    inner = H * D
    gemm = DIM * 4 * inner + DIM * DECAY_RANK + DECAY_RANK * inner + DIM * H + inner * DIM
    layer = sum(KERNEL_FLOPS_PER_TOKEN_HEAD.values()) * H
    return 3 * 2 * gemm + layer


def bench_mixer(a, rank, world, local_rank):
    import torch.distributed as dist
    from sophia_b200 import _lib, dp
    from sophia_b200.mixer import KDAMixerBlock

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    B = a.batch or 4
    gen = torch.Generator().manual_seed(42 + rank)
    m = KDAMixerBlock(dim=DIM, heads=H, decay_rank=DECAY_RANK, generator=gen).to(device)
    x = torch.randn(B, T, DIM, generator=gen).to(device, torch.bfloat16)
    dout = torch.randn(B, T, DIM, generator=gen).to(device, torch.bfloat16)
    params = list(m.parameters())
    layer = {"A_log": m.A_log, "dt_bias": m.dt_bias, "conv_q": m.conv_q, "conv_k": m.conv_k, "conv_v": m.conv_v}
    flat = torch.empty(sum(p.numel() for p in params), device=device, dtype=torch.float32)
    small = torch.empty(dp.bucket_numel(H, D), device=device, dtype=torch.float32)

    def step(xin=None, din=None):
        for prm in params:
            prm.grad = None
        xx = (x if xin is None else xin).detach().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = m(xx)
        out.backward(dout if din is None else din)
        if world > 1:  # data parallel: one all-reduce of every weight gradient
            torch.cat([prm.grad.reshape(-1) for prm in params], out=flat)
            dist.all_reduce(flat)
        dp.grad_bucket(layer, out=small)
        return small

    def timed(fn, steps, sampler=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        if sampler is not None:
            sampler.mark(h0, time.perf_counter())
        if world > 1:
            dist.barrier()
        return dp.max_over_ranks(e0.elapsed_time(e1), device)

    for _ in range(a.warmup):
        step()
    if a.profile:
        timed(step, a.steps)
        return None
    sampler = ClockSampler(device)
    sampler.start()
    ms = timed(step, a.steps, sampler)
    clocks = sampler.stop()
    tokens = world * B * T * a.steps
    value = tokens / (ms / 1e3)

    _lib.timing_reset()
    _lib.timing_enable(True)
    timed(step, a.steps)
    _lib.timing_enable(False)
    kern = _lib.timing_read()
    _lib.timing_reset()
    launches = sum(n for n, _ in kern.values())

    # end to end: x and dO cross from pinned host memory every step (two
    # alternating buffers on a copy stream), the layer's small weight
    # gradients come back
    host = {"x": x.detach().cpu().pin_memory(), "do": dout.detach().cpu().pin_memory()}
    bufs = [{k: torch.empty_like(v, device=device) for k, v in host.items()} for _ in range(2)]
    out_host = torch.empty(small.numel(), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(device=device)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(steps):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        copy_stream.wait_event(e0)

        def issue_copy(i):
            b = i % 2
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(freed[b])
                for k in host:
                    bufs[b][k].copy_(host[k], non_blocking=True)
                copied[b].record(copy_stream)

        issue_copy(0)
        for i in range(steps):
            if i + 1 < steps:
                issue_copy(i + 1)
            b = i % 2
            st.wait_event(copied[b])
            step(bufs[b]["x"], bufs[b]["do"])
            out_host.copy_(small, non_blocking=True)
            freed[b].record(st)
        e1.record(st)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return dp.max_over_ranks(e0.elapsed_time(e1), device)

    e2e_run(2)
    e2e_steps = max(3, min(a.steps, 10))
    ms_e2e = e2e_run(e2e_steps)

    hbm, tc, tc_sus, src = peaks()
    th = B * T * H
    dom = max((k for k in kern if k in KERNEL_BYTES_PER_TOKEN_HEAD), key=lambda k: kern[k][1])
    n_l, tot = kern[dom]
    achieved = KERNEL_BYTES_PER_TOKEN_HEAD[dom] * th / (tot / max(1, n_l) / 1e3) / 1e9
    block_tflops = mixer_flops_per_token() * B * T / (ms / a.steps / 1e3) / 1e12
    return {
        "value": value, "ms": ms / a.steps, "B": B, "clocks": clocks,
        "e2e": {"value": world * B * T * e2e_steps / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host.values()),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None, "peak_source": src,
                     "block": {"bound": "tensor", "flops_per_token": round(mixer_flops_per_token()),
                               "achieved_tflops": round(block_tflops, 1), "peak_tflops": tc_sus,
                               "frac": round(block_tflops / tc_sus, 4)},
                     "kernel_ms_per_step": {k: round(v[1] / a.steps, 4) for k, v in kern.items() if v[0]}},
    }


def cpu_block_sample(tokens: int):
    """The mixer block on the CPU in fp32 (torch ops around the oracle
    restatement of the reference recurrence), fwd+bwd on one sequence of
    `tokens` tokens.  Returns (tokens/s, seconds)."""
    sys.path.insert(0, ROOT)
    from torch.nn import functional as F
    from oracle.kda_oracle import kda_layer as oracle_layer
    from sophia_b200.mixer import KDAMixerBlock
    gen = torch.Generator().manual_seed(0)
    m = KDAMixerBlock(dim=DIM, heads=H, decay_rank=DECAY_RANK, generator=gen)
    x = torch.randn(1, tokens, DIM, generator=gen).requires_grad_(True)
    t0 = time.perf_counter()
    h = F.rms_norm(x, (DIM,), m.in_norm, m.eps)
    q, k, v, gate = F.linear(h, m.w_qkvg).split(H * D, dim=-1)
    decay = F.linear(F.linear(h, m.decay_down), m.decay_up)
    beta = F.linear(h, m.beta_proj)
    sh = (1, tokens, H, D)
    o = oracle_layer(q.reshape(sh), k.reshape(sh), v.reshape(sh), decay.reshape(sh), beta, m.A_log, m.dt_bias,
                     conv_weights=[m.conv_q, m.conv_k, m.conv_v], compute_dtype=torch.float32).o
    y = F.rms_norm(o, (D,), m.out_norm, m.eps) * torch.sigmoid(gate.reshape(sh))
    out = F.linear(y.reshape(1, tokens, H * D), m.o_proj)
    out.square().mean().backward()
    dt = time.perf_counter() - t0
    return tokens / dt, dt


def dp_shard(n, rank, world):
    from sophia_b200.dp import shard
    return shard(n, rank, world)


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    mixer = a.workload == "cfg2"
    decode = a.workload == "decode"
    metric = MIXER_METRIC if mixer else (DECODE_METRIC if decode else METRIC)
    config = {"workload": a.workload, "global_batch": (a.batch or 8) * world if a.workload == "cfg1" else 320,
              "seq_len": T, "heads": H, "head_dim": D, "chunk": 64,
              "parallelism": f"dp{world}", "l2": "inputs larger than L2 (128 MiB per tensor), no flush"}
    if a.workload == "cfg4":
        ncu4 = len(cfg4_cu_seqlens()) - 1
        config.update({"global_batch": world, "seq_len": CFG4_WINDOWS * T,
                       "packing": f"{CFG4_WINDOWS} windows x {T} tokens, {ncu4} documents (log-uniform lengths in "
                                  "[32, 4096], seed 42), cu_seqlens int32 built on the device from the windows' "
                                  f"end-of-document tokens every step (capacity {CFG4_CAPACITY}), state and conv "
                                  "history reset per document"})
    if a.workload == "cfg3":
        per_rank = len(range(CFG3_SEQS)[dp_shard(CFG3_SEQS, rank, world)])
        config.update({"global_batch": CFG3_SEQS, "micro_batch": min(per_rank, CFG3_MICRO),
                       "update": f"{CFG3_SEQS} sequences per update, {per_rank} on rank 0 in micro-batches of at most "
                                 f"{CFG3_MICRO}, weight gradients accumulated, one all-reduce"})
    if world > 1:
        config["all_reduce"] = "asynchronous: overlaps the next step's compute; the timed region waits for the last"
    if mixer:
        config.update({"global_batch": (a.batch or 4) * world, "hidden": DIM, "decay_rank": DECAY_RANK,
                       "l2": "activations larger than L2 (48 MiB input, 256 MiB projections), no flush"})
    if decode:
        Bd = a.batch or DECODE_BATCH
        config.update({"global_batch": Bd * world, "seq_len": 1, "chunk": None,
                       "step": "one kda_decode call: one token for each sequence (ShortConv with its history + "
                               "the recurrence), state and conv history carried",
                       "l2": (f"fp32 states ({Bd * H * D * D * 4 >> 20} MiB) "
                              + ("larger than L2, no flush" if Bd * H * D * D * 4 > 126e6 else "fit in L2"))})
        if world > 1:
            config["all_reduce"] = None
    sample = cpu_block_sample if mixer else cpu_sample
    what = "mixer block (torch fp32 ops around the oracle recurrence)" if mixer else \
        "16 heads (oracle restatement of the reference CPU path, torch fp32 autograd)"
    if a.impl == "reference" and decode:
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        Bd = a.batch or DECODE_BATCH
        cpu_decode_sample(Bd, max(a.warmup, 1), threads)
        rate, secs = cpu_decode_sample(Bd, a.steps, threads)
        config["cpu_sample"] = f"each step: one token for {Bd} sequences x {H} heads on the host (no conv history)"
        line = {"metric": metric, "value": rate, "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": secs / a.steps * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": f"{a.steps} decode steps of {Bd} sequences (oracle restatement of the "
                                           "reference recurrence, fp32)"},
                "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if a.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        sample_tokens = 256 if mixer else CPU_SAMPLE_TOKENS
        for _ in range(a.warmup):
            sample(64)
        rates, secs = [], 0.0
        for _ in range(a.steps):
            r, dt = sample(sample_tokens)
            rates.append(r)
            secs += dt
        value = sample_tokens * a.steps / secs
        config["cpu_sample"] = f"each step: 1 sequence x {sample_tokens} tokens x {H} heads fwd+bwd on the host"
        line = {"metric": metric, "value": value, "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": secs / a.steps * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": f"1 sequence x {sample_tokens} tokens fwd+bwd per step, {what}"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    res = (bench_mixer if mixer else (bench_decode if decode else bench_ours))(a, rank, world, local_rank)
    if res is None:  # --profile
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    cpu = None
    if rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        if decode:
            Bd = a.batch or DECODE_BATCH
            cpu_decode_sample(Bd, 1, threads)  # warm-up
            n_s, dt = 0, 0.0
            while n_s < 3 or dt < 5.0:
                _, d = cpu_decode_sample(Bd, 1, threads)
                dt += d
                n_s += 1
                if dt > 20.0:
                    break
            cpu = {"value": Bd * n_s / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                   "sample": f"{n_s} decode steps of {Bd} sequences x {H} heads ({dt:.1f} s; oracle restatement "
                             "of the reference recurrence, fp32, no conv history)"}
        elif mixer:
            torch.set_num_threads(threads)
            rate, dt = cpu_block_sample(1024)
            n_s, tok = 1, 1024
        else:
            cpu_sample(64, threads)  # warm-up
            n_s, tok, dt = 0, CPU_SAMPLE_TOKENS, 0.0
            while n_s < 3 or dt < 10.0:  # 10-30 s of CPU work
                _, d = cpu_sample(tok, threads)
                dt += d
                n_s += 1
                if dt > 30.0:
                    break
            rate = n_s * tok / dt
        if not decode:
            cpu = {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                   "sample": f"{n_s} x (1 sequence x {tok} tokens fwd+bwd) ({dt:.1f} s), {what}"}
    if rank == 0:
        line = {"metric": metric, "value": res["value"], "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": res["ms"], "higher_is_better": True,
                "scaling": "strong" if a.workload == "cfg3" else "weak", "vs_baseline": None,
                "dtype": "f32" if decode else "bf16",
                "data": "synthetic", "config": config, "roofline": res["roofline"], "cpu_baseline": cpu,
                "e2e": res["e2e"], "gpu_launches": res["gpu_launches"], "clocks": res["clocks"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
