"""Headline benchmark: bulk Qwen3-0.6B-architecture embedding (bf16), config 5.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the config-5 corpus (65,536 seeded texts, lognormal lengths clipped
to [8, 2048]), longest-first and packed into varlen batches of at most 65,536
real tokens. One step = one packed batch through the full 28-layer tower,
last-token pooling and L2 on one GPU. Under torchrun each rank is an
independent replica on its own GPU taking every N-th batch (weak scaling, no
collective on the data path; NCCL only for the barrier and the max-over-ranks
time). ``value`` = real tokens of all ranks / max over ranks of the device
time of K steps with ids already in HBM; ``e2e`` = the same through the public
API with pinned host ids and host outputs, copies inside the timed region.

``--impl reference`` times the CPU reference arm on the host cores: the
torch-CPU f32 (MKL) restatement of the reference's forward
(oracle/qwen3_torch.py, pinned to the numpy restatement oracle/qwen3.py), each
step a bounded sample of the same corpus; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "embedded tokens/sec (Qwen3-0.6B arch, bf16)"
BATCH_TOKENS = 65536
N_TEXTS = 65536
CPU_SAMPLE_TOKENS = 8192  # tokens of one CPU-baseline sample (10-30 s of CPU work)
REF_TIME_BUDGET_S = 150.0  # CPU seconds the reference arm's timed steps may take together
REF_MIN_SAMPLE_TOKENS = 256
REF_MAX_SAMPLE_TOKENS = 8192


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops_sustained") or d.get("bf16_tflops"), "measured"
    return 1400.0, "fallback"


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of one GPU, sampled
    in-process through NVML every 100 ms while the timed region runs (the same
    fields as `nvidia-smi --query-gpu=clocks.sm,clocks.max.sm,power.draw,
    clocks_event_reasons.*`, without spawning a process per sample)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.sm: list[float] = []
        self.reasons: set = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._h = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(cuda_index)
            bus = getattr(props, "pci_bus_id", None)
            dom = getattr(props, "pci_domain_id", 0)
            dev = getattr(props, "pci_device_id", 0)
            if bus is not None:
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0".encode())
            else:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self._nv = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._h = None

    def _run(self):
        nv = getattr(self, "_nv", None)
        while not self._stop.is_set() and self._h is not None:
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)))
                try:
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml"}


def corpus_batches():
    import im_not_llm_b200 as inl

    lengths, ids = inl.synthetic.cfg5_corpus(n_texts=N_TEXTS)
    order = inl.planner.longest_first(lengths)
    texts = np.split(ids, np.cumsum(lengths)[:-1])
    plan = inl.planner.plan_packed([lengths[i] for i in order], BATCH_TOKENS)
    batches = [[order[k] for k in r] for r in plan]
    return texts, batches, lengths


def cpu_sample(texts, lengths, budget_tokens: int, seed: int):
    """A bounded CPU sample of the corpus: texts drawn uniformly at random
    (long ones included, so the sample keeps the corpus's length mix) until
    about ``budget_tokens`` real tokens; packed as (ids, cu, texts, tokens)."""
    rng = np.random.default_rng(seed)
    picked, total = [], 0
    for i in rng.permutation(len(texts)):
        picked.append(int(i))
        total += int(lengths[i])
        if total >= budget_tokens:
            break
    ids = np.concatenate([texts[i] for i in picked])
    cu = np.zeros(len(picked) + 1, dtype=np.int32)
    np.cumsum([lengths[i] for i in picked], out=cu[1:])
    return ids, cu, len(picked), total


def cpu_reference_rate(cpu_model, texts, lengths, budget_tokens=CPU_SAMPLE_TOKENS, seed=0):
    """Tokens/s of the torch-CPU f32 restatement (oracle/qwen3_torch.py, MKL
    on every host thread) on a bounded sample of the corpus."""
    ids, cu, n, total = cpu_sample(texts, lengths, budget_tokens, seed)
    t0 = time.perf_counter()
    cpu_model.embed_last(ids, cu)
    dt = time.perf_counter() - t0
    return total / dt, total, n, dt


def cpu_model(weights, cfg):
    import torch

    from oracle import qwen3_torch as QT

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return QT.Qwen3Cpu(weights, cfg), threads


def rank_share(batches: list, costs: list, rank: int, world: int, steps: int, warmup: int) -> list:
    """The batches one rank runs, warm-up first. The corpus's batches are
    dealt to the ranks longest-processing-time first on their forward cost
    (``planner.assign_lpt`` over ``planner.batch_cost``), so every rank holds
    about the same work and no rank always draws the heaviest batch. The
    timed steps are the rank's whole share when ``steps`` covers it, else
    ``steps`` batches spaced evenly over the share in descending cost (a
    prefix would over-weight the attention-heavy 2k-token texts); the warm-up
    batches come from the same spread."""
    import im_not_llm_b200 as inl

    share = inl.planner.assign_lpt(costs, world)[rank]  # heaviest first
    mine = [batches[b] for b in share]
    if steps >= len(mine):
        timed = [mine[i % len(mine)] for i in range(steps)]
    else:
        timed = [mine[int(i)] for i in np.linspace(0, len(mine) - 1, steps)]
    return [timed[i % len(timed)] for i in range(warmup)] + timed


def reduce_timing(ms: float, e2e_ms: float, tokens: float, world: int, device: str) -> tuple[float, float, float]:
    """Across ranks: the max of the device-timed and the end-to-end times,
    the sum of the tokens (every rank takes the same collective steps)."""
    if world == 1:
        return ms, e2e_ms, float(tokens)
    import torch
    import torch.distributed as dist

    stats = torch.tensor([ms, e2e_ms, float(tokens)], dtype=torch.float64, device=device)
    mx = stats.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    tot = stats.clone()
    dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    return mx[0].item(), mx[1].item(), tot[2].item()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args, world, rank):
    if rank != 0:
        return
    import im_not_llm_b200 as inl

    cfg = dict(inl.synthetic.QWEN3_0_6B)
    weights = inl.synthetic.qwen3_weights(cfg, seed=0)
    texts, _, lengths = corpus_batches()
    model, threads = cpu_model(weights, cfg)
    # The warm-up samples (at least one) also measure this host's rate; each
    # timed step's sample is then sized so all steps fit REF_TIME_BUDGET_S.
    rate = 0.0
    for w in range(max(args.warmup, 1)):
        rate = cpu_reference_rate(model, texts, lengths, budget_tokens=512, seed=100 + w)[0]
    per_step = int(np.clip(rate * REF_TIME_BUDGET_S / max(args.steps, 1), REF_MIN_SAMPLE_TOKENS, REF_MAX_SAMPLE_TOKENS))
    toks, secs = 0, 0.0
    for s in range(args.steps):
        _, n, _, dt = cpu_reference_rate(model, texts, lengths, budget_tokens=per_step, seed=s)
        toks += n
        secs += dt
    value = toks / secs
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "cfg5 corpus, bounded CPU sample per step", "sample_tokens_per_step": toks // max(args.steps, 1)},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} samples of ~{per_step} tokens of the cfg5 corpus (texts drawn "
                                   f"uniformly, long ones included; sized from the warm-up rate to fit "
                                   f"{REF_TIME_BUDGET_S:.0f} s), torch-CPU f32 restatement of "
                                   f"crates/inl-text/src/qwen3/mod.rs (MKL) on {threads} threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def run_ours(args, world, rank, local):
    import torch

    import im_not_llm_b200 as inl

    torch.cuda.set_device(local)
    cfg = dict(inl.synthetic.QWEN3_0_6B)
    weights = inl.synthetic.qwen3_weights(cfg, seed=0)
    model = inl.CudaModel(cfg, weights, device=local, dtype="bf16")
    texts, batches, lengths = corpus_batches()
    need = args.warmup + args.steps
    costs = [inl.planner.batch_cost([lengths[i] for i in b]) for b in batches]
    sel = rank_share(batches, costs, rank, world, args.steps, args.warmup)
    packed = [inl.planner.pack(texts, b) for b in sel]
    # inputs resident in HBM for the device-timed leg
    dev_ids = [torch.from_numpy(p[0].view(np.int32)).cuda() for p in packed]
    max_n = max(len(b) for b in sel)
    dev_out = torch.empty(max_n, cfg["hidden_size"], dtype=torch.float32, device="cuda")
    stream = torch.cuda.ExternalStream(model.stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    for i in range(args.warmup):
        model.embed(dev_ids[i].data_ptr(), packed[i][1], out=dev_out.data_ptr())
    torch.cuda.synchronize()

    # ---------------- device-timed leg (value): no per-launch events inside
    model.launch_count(reset=True)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = 0
    barrier()
    torch.cuda.synchronize()
    step_ms = []
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k, i in enumerate(range(args.warmup, need)):
            t0 = time.perf_counter()
            step_ev[k][0].record(stream)
            model.embed(dev_ids[i].data_ptr(), packed[i][1], out=dev_out.data_ptr())
            step_ev[k][1].record(stream)
            step_ms.append(round((time.perf_counter() - t0) * 1000.0, 2))
            tokens += int(packed[i][1][-1])
        stop.record(stream)
        torch.cuda.synchronize()
    step_dev_ms = [round(a.elapsed_time(b), 2) for a, b in step_ev]
    barrier()
    ms = start.elapsed_time(stop)
    launches = model.launch_count()

    # ---------------- profiled pass (roofline): the same steps again, with CUDA
    # events around every GEMM and attention launch on the model's stream
    model.set_profiling(True)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for i in range(args.warmup, need):
        model.embed(dev_ids[i].data_ptr(), packed[i][1], out=dev_out.data_ptr())
    p1.record(stream)
    torch.cuda.synchronize()
    prof_step_ms = p0.elapsed_time(p1)
    prof = model.profile(-1)
    kinds = {name: model.profile(k) for k, name in enumerate(("qkv", "o", "gate_up", "down"))}
    attn_prof = model.profile(100)  # attention launches
    model.set_profiling(False)

    # ---------------- end-to-end leg (e2e): pinned host ids -> host embeddings
    host_ids = []
    for p in packed:
        t = torch.empty(len(p[0]), dtype=torch.int32).pin_memory()
        t.numpy()[:] = p[0].view(np.int32)
        host_ids.append(t.numpy().view(np.uint32))
    host_out = torch.empty(max_n, cfg["hidden_size"], dtype=torch.float32).pin_memory().numpy()
    h2d = d2h = 0
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.warmup, need):
        n = len(packed[i][1]) - 1
        model.embed(host_ids[i], packed[i][1], out=host_out[:n])
        h2d += host_ids[i].nbytes + packed[i][1].nbytes
        d2h += n * cfg["hidden_size"] * 4
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()

    ms_max, e2e_max, tokens_all = reduce_timing(ms, e2e_s * 1000.0, tokens, world, "cuda")

    if rank == 0:
        peak, peak_kind = _peaks()
        achieved = prof["flops"] / (prof["ms"] / 1000.0) / 1e12 if prof["ms"] > 0 else 0.0
        line = {
            "metric": METRIC, "value": tokens_all / (ms_max / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded cfg5 corpus (lognormal lengths, uniform ids), random-init N(0,0.02) weights",
            "config": {"workload": "cfg5 bulk Qwen3-0.6B last-token embedding, packed varlen batches",
                       "batch_tokens": BATCH_TOKENS, "corpus_texts": N_TEXTS,
                       "tokens_per_step_per_gpu": tokens / args.steps,
                       "l2": "no flush: working set per step > L2 (1.2 GB bf16 weights, >=128 MB activations)",
                       "parallelism": f"dp{world} independent replicas"},
            "roofline": {"bound": "tensor", "kernel": "tcgen05 GEMMs of all projections (gemm_bf16_tn: qkv; gemm_bf16_pair: o, gate/up, down)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} bf16 sustained",
                         "traffic": GEMM_TRAFFIC_BYTES_PER_LAUNCH,
                         "traffic_source": "fixed figure from one ncu capture of a config-5 step (mean "
                                           "dram__bytes_read.sum + dram__bytes_write.sum per GEMM launch), "
                                           "not measured by this run; algorithmic bytes per launch ~6.1e8",
                         "timing": "per-launch CUDA events in a second pass over the same steps; value is "
                                   "timed without them",
                         "gemm_launches": prof["launches"], "gemm_ms": prof["ms"],
                         "gemm_share_of_step": prof["ms"] / prof_step_ms if prof_step_ms > 0 else None,
                         "attention_ms_per_step": attn_prof["ms"] / args.steps,
                         "attention_share_of_step": attn_prof["ms"] / prof_step_ms if prof_step_ms > 0 else None,
                         "by_projection": {k: {"ms_per_step": v["ms"] / args.steps,
                                               "tflops": v["flops"] / (v["ms"] / 1000.0) / 1e12 if v["ms"] else 0.0}
                                           for k, v in kinds.items()}},
            "e2e": {"value": tokens_all / (e2e_max / 1000.0), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps},
            "gpu_launches": launches,
            "host_step_ms": step_ms,
            "device_step_ms": step_dev_ms,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            cm, threads = cpu_model(weights, cfg)
            cpu_reference_rate(cm, texts, lengths, budget_tokens=256, seed=99)  # warm-up
            r, n, k, dt = cpu_reference_rate(cm, texts, lengths)
            line["cpu_baseline"] = {"value": r, "unit": "tokens/s", "cores": threads, "kind": "port",
                                    "sample": f"{k} texts / {n} tokens of the cfg5 corpus (drawn uniformly) through "
                                              f"the torch-CPU f32 restatement (oracle/qwen3_torch.py, MKL) on "
                                              f"{threads} threads, {dt:.1f}s"}
        emit(line)
    model.close()


# Mean DRAM bytes (read + write) per GEMM launch (gemm_bf16_tn_kernel for QKV,
# gemm_bf16_pair_kernel for o, gate/up and down) over one config-5 bench step
# (64.6k tokens), measured with ncu: 465.4 MB.
GEMM_TRAFFIC_BYTES_PER_LAUNCH = 465.4e6

KERNEL_CASES = {
    # name: (M tokens, N, K, epilogue) — the four projections of one Qwen3-0.6B layer
    "gemm_qkv": (32768, 4096, 1024, 0),
    "gemm_o": (32768, 1024, 2048, 1),
    "gemm_gateup": (32768, 6144, 1024, 2),
    "gemm_down": (32768, 1024, 3072, 1),
}


def run_kernel_case(name: str, reps: int = 3):
    """A single kernel on a small case (a few hundred MB on the device), for
    ncu captures and quick timing: `python bench.py --case gemm_gateup`."""
    import ctypes

    import torch

    from im_not_llm_b200 import _native as N

    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")  # device wait status of the GEMM cases
    if name in ("gemm_qkv_fused", "gemm_gateup_fused"):
        M, K = 32768, 1024
        fused_qkv = name == "gemm_qkv_fused"
        Nn = 4096 if fused_qkv else 6144
        A = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
        W = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
        out = torch.empty(M, Nn if fused_qkv else Nn // 2, device="cuda", dtype=torch.bfloat16)
        ss = torch.rand(M, K // 64, device="cuda") + 1.0
        pos = (torch.arange(M, device="cuda", dtype=torch.int32) % 2048)  # packed texts: consecutive positions
        cs = torch.rand(32, 2048, 4, device="cuda")  # RoPE pairs [d/4, max_pos, (cos, cos, sin, sin)]
        qn = torch.ones(128, device="cuda")
        a = N.GemmEx()
        a.A, a.lda, a.W, a.ldw, a.M, a.N, a.K = A.data_ptr(), K, W.data_ptr(), K, M, Nn, K
        a.epi, a.act, a.gate_block = (4 if fused_qkv else 2), 0, 128
        a.out, a.ldo = out.data_ptr(), out.stride(0)
        a.ss_in, a.ss_in_parts, a.ss_dim, a.ss_eps = ss.data_ptr(), K // 64, K, 1e-6
        a.status = status.data_ptr()
        if fused_qkv:
            a.qn = a.kn = qn.data_ptr()
            a.pos, a.cos = pos.data_ptr(), cs.data_ptr()
            a.hq, a.hkv, a.d, a.max_pos, a.qk_eps = 16, 8, 128, 2048, 1e-6

        def launch():
            N.check(N.lib().inl_cuda_gemm_bf16_ex(ctypes.byref(a), s), name)
        flops = 2.0 * M * Nn * K
    elif name.startswith("gemm"):
        M, Nn, K, epi = KERNEL_CASES[name]
        A = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
        W = (torch.randn(Nn, K, device="cuda") * 0.02).to(torch.bfloat16)
        out = torch.empty(M, Nn // 2 if epi == 2 else Nn, device="cuda", dtype=torch.bfloat16)
        resid = out if epi == 1 else None

        def launch():
            N.check(N.lib().inl_cuda_gemm_bf16(A.data_ptr(), K, W.data_ptr(), K, M, Nn, K, epi, 0, 128,
                                               out.data_ptr(), out.stride(0),
                                               None if resid is None else resid.data_ptr(), out.stride(0), 0,
                                               status.data_ptr(), s), name)
        flops = 2.0 * M * Nn * K
    elif name in ("attention", "attention_cfg5"):
        if name == "attention":
            lengths = [2048] * 4 + [512] * 8 + [256] * 16
        else:  # ~64k tokens of config 5's lognormal lengths, in corpus order (seeded)
            import im_not_llm_b200 as inl

            all_lengths, _ = inl.synthetic.cfg5_corpus(n_texts=1024)
            lengths = []
            for L in all_lengths:
                if sum(lengths) + int(L) > 65536:
                    break
                lengths.append(int(L))
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        T = int(cu[-1])
        qkv = torch.randn(T, 4096, device="cuda").to(torch.bfloat16)
        o = torch.empty(T, 2048, device="cuda", dtype=torch.bfloat16)

        def launch():
            N.check(N.lib().inl_cuda_attention(qkv.data_ptr(), qkv.data_ptr() + 2048 * 2, qkv.data_ptr() + 3072 * 2,
                                               4096, 4096, 4096, o.data_ptr(), 2048, 1, 16, 8, 128, 128 ** -0.5, 1,
                                               -1, cu.ctypes.data, len(lengths), s), name)
        flops = sum(4.0 * 2048 * L * (L + 1) / 2 for L in lengths)
    elif name in ("norm", "layer_norm", "qk_norm_rope_d256"):
        # HBM-bound row kernels at config sizes larger than L2: RMSNorm / LayerNorm
        # over 65536 x 1024 bf16 rows (Qwen3 width), and config 4's q / k / v norm
        # + RoPE over 66k tokens x (3 + 1 + 1) heads of 256 (v weightless)
        if name == "qk_norm_rope_d256":
            T, hq, hkv, d = 66142, 3, 1, 256
            ld = (hq + 2 * hkv) * d
            qkv = torch.randn(T, ld, device="cuda").to(torch.bfloat16)
            qw, kw = torch.ones(d, device="cuda"), torch.ones(d, device="cuda")
            pos = (torch.arange(T, device="cuda", dtype=torch.int32) % 2048)
            ang = torch.arange(2048, device="cuda", dtype=torch.float64)[:, None] / (1e6 ** (torch.arange(
                0, d // 2, device="cuda", dtype=torch.float64) * 2 / d))[None, :]
            cos, sin = ang.cos().float().contiguous(), ang.sin().float().contiguous()

            def launch():
                N.check(N.lib().inl_cuda_qk_norm_rope(qkv.data_ptr(), 1, ld, T, hq, hkv, d, qw.data_ptr(),
                                                      kw.data_ptr(), 1, 1e-6, pos.data_ptr(), cos.data_ptr(),
                                                      sin.data_ptr(), 2048, status.data_ptr(), s), name)
            nbytes = 2.0 * T * ld * 2
        else:
            rows, H = 65536, 1024
            x = torch.randn(rows, H, device="cuda").to(torch.bfloat16)
            y = torch.empty_like(x)
            wt = torch.rand(H, device="cuda") + 0.5
            bias = torch.zeros(H, device="cuda")
            ln = 1 if name == "layer_norm" else 0

            def launch():
                N.check(N.lib().inl_cuda_norm(x.data_ptr(), 1, H, wt.data_ptr(), bias.data_ptr() if ln else None,
                                              1e-6, ln, rows, H, y.data_ptr(), 1, H, s), name)
            nbytes = 2.0 * rows * H * 2
        flops = 0.0
    elif name == "attention_cfg4":
        # config 4's attention: 128 texts of log-uniform lengths (seed 4), 3 query
        # heads / 1 K/V head x 256, bidirectional, the 512-token window of 5 in 6 layers
        import im_not_llm_b200 as inl

        _, cu = inl.synthetic.cfg4_inputs()
        cu = np.ascontiguousarray(cu, dtype=np.int32)
        lengths = np.diff(cu)
        T, hq, hkv, d, win = int(cu[-1]), 3, 1, 256, 512
        ld = (hq + 2 * hkv) * d
        qkv = torch.randn(T, ld, device="cuda").to(torch.bfloat16)
        o = torch.empty(T, hq * d, device="cuda", dtype=torch.bfloat16)

        def launch():
            N.check(N.lib().inl_cuda_attention(qkv.data_ptr(), qkv.data_ptr() + hq * d * 2,
                                               qkv.data_ptr() + (hq + hkv) * d * 2, ld, ld, ld, o.data_ptr(), hq * d,
                                               1, hq, hkv, d, 1.0, 0, win, cu.ctypes.data, len(lengths), s), name)
        # attended (query, key) pairs: |q - k| <= 512 inside each text
        pairs = 0.0
        for L in lengths:
            i = np.arange(int(L))
            pairs += float((np.minimum(i + win, L - 1) - np.maximum(i - win, 0) + 1).sum())
        flops = 4.0 * hq * d * pairs
    else:
        raise SystemExit(f"unknown case {name}")
    launch()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        launch()
    en.record()
    torch.cuda.synchronize()
    ms = st.elapsed_time(en) / reps
    code = int(status.item())
    rec = {"case": name, "ms": ms, "device_status": code}
    if flops:
        rec["tflops"] = flops / ms / 1e9
    else:  # HBM-bound: algorithmic bytes (each input read once, each output written once)
        hbm = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs") if (
            ROOT / "MEASURED_PEAKS.json").exists() else None
        rec["gb_per_s"] = nbytes / ms / 1e6
        rec["hbm_frac"] = rec["gb_per_s"] / hbm if hbm else None
    print(json.dumps(rec), flush=True)
    if code:
        raise SystemExit(f"{name}: a device wait ran past its limit (status {code})")


# The other BASELINE configurations, one forward of each config's own input
# per step: `python bench.py --case cfg2`. name: (architecture, dtype, output).
MODEL_CASES = {
    "cfg1": ("Qwen3-0.6B, 8 x 128 tokens, last-token pooling + L2", "f32", "dense"),
    "cfg2": ("ModernBERT SPLADE, 32 texts U[16, 256], V = 36282 max-pooled", "f32", "sparse"),
    "cfg3": ("Qwen3-0.6B bidirectional + 1024->128 per token, 64 x 512 tokens", "bf16", "late"),
    "cfg4": ("EmbeddingGemma-style, 128 texts log-U[32, 2048], mean pool + dense chain", "bf16", "dense"),
    "cfg2_bf16": ("ModernBERT SPLADE in bf16 (the decoder on the tcgen05 SEGMAX GEMM), config 2's texts", "bf16",
                  "sparse"),
    # the f32 configurations on the SIMT FFMA GEMMs instead of the 3xBF16 tensor-core GEMMs
    "cfg1_ffma": ("Qwen3-0.6B, 8 x 128 tokens, SIMT f32 GEMMs", "f32", "dense"),
    "cfg2_ffma": ("ModernBERT SPLADE, 32 texts, SIMT f32 GEMMs", "f32", "sparse"),
}


def run_model_case(name: str, reps: int = 10, warmup: int = 3):
    """Tokens/s of one configuration's full forward through the C ABI, ids
    and outputs resident on the device; GEMM and attention time from a
    second, profiled pass."""
    import torch

    import im_not_llm_b200 as inl

    S = inl.synthetic
    desc, dtype, kind = MODEL_CASES[name]
    ffma = name.endswith("_ffma")
    label = name
    name = name.removesuffix("_ffma").removesuffix("_bf16")
    if name == "cfg1":
        cfg, w = dict(S.QWEN3_0_6B), S.qwen3_weights(S.QWEN3_0_6B, seed=0)
        ids, cu = S.cfg1_inputs()
    elif name == "cfg2":
        cfg, w = dict(S.MODERNBERT_SPLADE), S.modernbert_weights(S.MODERNBERT_SPLADE, seed=0)
        ids, cu = S.cfg2_inputs()
    elif name == "cfg3":
        cfg, w = dict(S.QWEN3_0_6B, is_causal=False), S.qwen3_weights(S.QWEN3_0_6B, seed=0)
        ids, cu = S.cfg3_inputs()
    else:
        cfg, w = dict(S.GEMMA_STYLE), S.gemma_weights(S.GEMMA_STYLE, seed=0)
        ids, cu = S.cfg4_inputs()
    m = inl.CudaModel(cfg, w, dtype=dtype)
    if name == "cfg3":
        m.set_dense_head(S.late_projection(cfg))
    if ffma:
        m.set_f32_gemm("ffma")
    info = m.info()
    T, n = int(cu[-1]), len(cu) - 1
    dev_ids = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.uint32).view(np.int32)).cuda()
    rows, cols = {"dense": (n, info["dense_dim"]), "sparse": (n, info["sparse_dim"]),
                  "late": (T, info["multivector_dim"])}[kind]
    out = torch.empty(rows, cols, dtype=torch.float32, device="cuda")
    fwd = {"dense": m.embed, "sparse": m.encode_sparse, "late": m.encode_multivector}[kind]

    def step():
        fwd(dev_ids.data_ptr(), cu, out=out.data_ptr())

    for _ in range(warmup):
        step()
    stream = torch.cuda.ExternalStream(m.stream)
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record(stream)
    for _ in range(reps):
        step()
    en.record(stream)
    torch.cuda.synchronize()
    ms = st.elapsed_time(en) / reps
    m.set_profiling(True)
    for _ in range(reps):
        step()
    torch.cuda.synchronize()
    g, a = m.profile(-1), m.profile(100)
    m.set_profiling(False)
    m.close()
    print(json.dumps({"case": label, "workload": desc, "dtype": dtype, "tokens": T, "texts": n, "ms": ms,
                      "tokens_per_s": T / (ms / 1000.0),
                      "gemm_tflops": g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] else None,
                      "gemm_ms": g["ms"] / reps, "attention_ms": a["ms"] / reps,
                      "note": "inputs and outputs resident on the device; GEMM / attention times from a "
                              "second pass with per-launch events"}), flush=True)


# The benchmark's stdout carries exactly one JSON line. main() keeps the real
# stdout here and points file descriptor 1 at stderr, so whatever a library
# prints there (NCCL's version banner under torchrun, for one) goes to stderr.
_JSON_OUT = None


def emit(line: dict) -> None:
    print(json.dumps(line), file=_JSON_OUT or sys.stdout, flush=True)


def main():
    global _JSON_OUT
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(KERNEL_CASES) + sorted(MODEL_CASES) +
                    ["attention", "attention_cfg5", "attention_cfg4", "gemm_qkv_fused", "gemm_gateup_fused", "norm",
                     "layer_norm", "qk_norm_rope_d256"],
                    default=None,
                    help="time one kernel on a small case instead of the benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.case in MODEL_CASES:
        run_model_case(args.case)
        return
    if args.case:
        run_kernel_case(args.case)
        return
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
