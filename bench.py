"""bs=1 greedy decode throughput of Llama-2-7B Q4_K_M on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step is one decode token (all 32 layers + LM head + argmax) of a random-init
Llama-2-7B Q4_K_M GGUF (seeded; weights 4.07 GB/token >> 126 MB L2, so no L2
flush is needed between steps), after a 128-token uniform-random prompt.
N > 1 is tensor parallel (strong scaling: one token stream per job); the ranks
exchange partial sums inside the step kernel over NVLink peer memory.

value   = tokens/s of the job, device-timed with CUDA events on the engine's
          stream over K device-fed graph launches (max over ranks).
e2e     = the same through the public per-step API (af_engine_step) over the
          same positions: each step copies the token id host->device and reads
          the next id back (host wall clock, max over ranks).
roofline: dominant kernel = the persistent step kernel (one launch per token);
          algorithmic bytes (weights + KV rows read) per launch / its
          event-timed duration, vs the measured HBM copy peak.
cpu_baseline: the reference's own CPU decode (oracle/_ref, compiled from the
          unmodified sources), production Q8_0 path, all host threads, on a
          bounded sample of decode steps.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 128
SEED = 0

# DRAM bytes (read + write) of one step_kernel launch, measured by ncu on the
# full workload (dram__bytes_read.sum + dram__bytes_write.sum, one pass; launch
# 132 of `python bench.py --steps 3 --warmup 3 --no-cpu-baseline`, context
# 132, single B200): 4.22 GB read + 5.77 MB written, 1.003x the algorithmic
# bytes.  Reported as roofline.traffic for that workload only.
STEP_KERNEL_DRAM_BYTES = {("llama2-7b", 1): 4_225_770_000}


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        for ln in open(self.f.name).read().splitlines():
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) >= 8:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def model_file(preset: str, rank: int, dist) -> str:
    from llm_core_b200 import gguf
    d = os.environ.get("AF_BENCH_DIR")
    if not d:
        need = gguf.model_weight_bytes(gguf.PRESETS[preset]) * 1.2
        d = tempfile.gettempdir()
        try:
            st = os.statvfs("/dev/shm")
            if st.f_bavail * st.f_frsize > need * 1.5:
                d = "/dev/shm"
        except OSError:
            pass
    path = os.path.join(d, f"af_bench_{preset}_s{SEED}.gguf")
    if rank == 0 and not os.path.exists(path):
        gguf.write_random_model(path, preset, SEED)
    if dist is not None:
        dist.barrier()
    return path


class _QuietStdout:
    """The reference library prints a banner on stdout when its backend
    initialises; keep the bench's stdout to the one JSON line."""

    def __enter__(self):
        sys.stdout.flush()
        self.fd = os.dup(1)
        devnull = os.open(os.devnull, os.O_WRONLY)
        os.dup2(devnull, 1)
        os.close(devnull)

    def __exit__(self, *a):
        os.dup2(self.fd, 1)
        os.close(self.fd)


def open_ref(path: str, threads: int):
    from oracle import RefLib
    with _QuietStdout():
        return RefLib().open(path, threads=threads, f32_mode=False, max_ctx=4096)


def bench_prompt(vocab: int):
    """The 128-token uniform-random prompt both arms decode after (BOS first)."""
    rng = np.random.default_rng(1234)
    return [1] + rng.integers(0, vocab, PROMPT_LEN).tolist()


def set_prompt_len(n: int):
    """The prompt length of the run (--prompt-len: 128 for the 7B workload,
    32 for TinyLlama's, the KV length for Qwen2.5-3B's)."""
    global PROMPT_LEN
    PROMPT_LEN = n


def host_cpu() -> dict:
    """The host CPU the CPU numbers ran on: model name and the affinity mask."""
    model = "unknown"
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        aff = sorted(os.sched_getaffinity(0))
    except AttributeError:
        aff = list(range(os.cpu_count() or 1))
    # compress the mask into ranges, e.g. "0-63"
    parts, i = [], 0
    while i < len(aff):
        j = i
        while j + 1 < len(aff) and aff[j + 1] == aff[j] + 1:
            j += 1
        parts.append(f"{aff[i]}-{aff[j]}" if j > i else f"{aff[i]}")
        i = j + 1
    return {"cpu_model": model, "affinity": ",".join(parts), "threads": len(aff)}


L2_BYTES = 126 * 1024 * 1024


def l2_note(weight_bytes: int, scope: str) -> str:
    """The config's L2 statement: the weights streamed per step against the 126 MB L2."""
    gb = (f"{weight_bytes / 1e9:.2f} GB" if weight_bytes >= 1e9 else f"{weight_bytes / 1e6:.1f} MB") + f" weights per step{scope}"
    return f"inputs larger than L2 ({gb})" if weight_bytes > L2_BYTES else f"weights fit in L2 ({gb})"


def host_threads() -> int:
    """Host threads this process may run on (its affinity mask, not the machine's count)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def ref_decode_after_prompt(path: str, threads: int, vocab: int, warmup: int, steps: int):
    """The reference's own CPU path on the b200 arm's workload: prefill the
    same 128-token prompt (llama_forward_batch), `warmup` untimed decode
    steps, then `steps` timed ones — context PROMPT_LEN+1+warmup .. +steps.
    Returns (seconds, first timed position)."""
    prompt = bench_prompt(vocab)
    ref = open_ref(path, threads)
    lg = ref.forward_batch(prompt, 0)
    tok = int(np.argmax(lg))
    ref.time_decode(tok, warmup)
    p0 = len(prompt) + warmup
    secs = ref.time_decode(tok, steps)
    ref.close()
    return secs, p0


def cpu_baseline_sample(path: str, steps: int, threads: int, vocab: int, warmup: int) -> dict | None:
    """The reference CPU decode (production Q8_0 path) after the bench prompt."""
    from oracle import RefLib
    if not RefLib.available():
        return None
    secs, p0 = ref_decode_after_prompt(path, threads, vocab, warmup, steps)
    return {"value": steps / secs, "unit": "tok/s", "cores": threads, "kind": "reference",
            **host_cpu(),
            "sample": f"{steps} decode steps of the reference's own CPU path (Q8_0 activations, r8 repack, "
                      f"oracle/_ref built from the unmodified sources) at context {p0}..{p0 + steps} after "
                      f"the same 128-token prompt, {threads} threads, random-init Llama-2-7B Q4_K_M"}


def run_reference(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    from llm_core_b200 import gguf
    path = model_file(args.model, 0, None)
    threads = host_threads()
    from oracle import RefLib
    if not RefLib.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libaxref.so was not built "
                          "(reference sources absent when the repo was built)"}))
        return 0
    cfg = gguf.PRESETS[args.model]
    # the b200 arm's workload: the same prompt, then W untimed and K timed
    # decode tokens over the same context positions
    secs, p0 = ref_decode_after_prompt(path, threads, cfg.vocab, args.warmup, args.steps)
    val = args.steps / secs
    line = {
        "impl": "reference", "metric": "bs=1 decode tok/s", "value": round(val, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * secs / args.steps, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "q8_0-int8 dot + f32", "data": "synthetic (seeded random-init GGUF)",
        "config": {"workload": f"{cfg.name} Q4_K_M bs=1 greedy decode",
                   "model": cfg.name, "global_batch": 1, "seq_len": PROMPT_LEN,
                   "context": f"{p0}..{p0 + args.steps}",
                   "parallelism": "cpu threads",
                   "l2": l2_note(gguf.model_weight_bytes(cfg), "")},
        "cpu_baseline": {"value": round(val, 3), "unit": "tok/s", "cores": threads, "kind": "reference",
                         **host_cpu(),
                         "sample": f"{args.steps} decode steps at context {p0}..{p0 + args.steps} after the "
                                   "128-token prompt (production Q8_0 path, all host threads)"},
        "e2e": {"value": round(val, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_b200(args):
    import torch
    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        world = args.gpus if world == 1 and args.gpus == 1 else world
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from llm_core_b200 import gguf
    from llm_core_b200.engine import LlamaCudaModel, nccl_unique_id
    path = model_file(args.model, rank, dist)
    nid = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    t_load = time.time()
    m = LlamaCudaModel(path, device=local, tp_rank=rank, tp_size=world, nccl_id=nid)
    t_load = time.time() - t_load
    cfg = gguf.PRESETS[args.model]
    prompt = bench_prompt(cfg.vocab)
    # long prompts go through the batched prompt pass (single GPU); the timed
    # decode only depends on the context length they leave
    nxt, _ = m.prefill(prompt, 0, want_logits=False, batched=world == 1 and len(prompt) > 256)
    pos = len(prompt)
    stream = torch.cuda.ExternalStream(m.stream)
    # warm-up
    ids = m.decode_greedy(nxt, pos, args.warmup)
    tok = int(ids[-1]) if len(ids) else nxt
    pos += args.warmup
    clocks = ClockSampler(local)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    from llm_core_b200._lib import check
    check(m.lib.af_engine_decode_greedy(m.h, tok, pos, args.steps, None), "decode")
    ev1.record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    pos += args.steps
    ms_step = ms / args.steps
    value = 1000.0 / ms_step
    # e2e through the per-step public API (host token in, host id out), over
    # the same positions as the timed region (the KV rows there are simply
    # rewritten), so both numbers see the same attention context
    pos_e2e = pos - args.steps
    n_e2e = args.steps
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    t = tok
    for i in range(n_e2e):
        t, _ = m.step(t, pos_e2e + i, want_logits=False)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        tt = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    e2e = n_e2e / e2e_s
    # Roofline of the dominant kernel.  With the persistent step kernel (one
    # launch per token) that kernel is the whole step: its algorithmic bytes
    # are the weight stream plus the KV cache it reads, its launch time the
    # device-timed step above.  The separate-kernel path (tensor-parallel
    # ranks) is profiled per kernel with event-bracketed eager launches.
    peak, kind = peaks()
    wb = m.weight_bytes
    step_gbs = wb / (ms_step / 1e3) / 1e9
    ctx_mid = PROMPT_LEN + 1 + args.warmup + args.steps / 2
    kv_bytes = 2 * cfg.n_layer * ctx_mid * (cfg.n_kv_head // world) * (cfg.n_embd // cfg.n_head) * 4
    prof = m.profile(t, pos, 4)
    pos += 4
    if m.kernels_per_step == 1:
        kb = wb + kv_bytes
        k_us = 1000 * ms_step
        kname = f"step_kernel (1 launch/step; {kind} peak)"
    else:
        gem = [k for k in prof if k.startswith("gemv")]
        g_ms = sum(prof[k]["ms"] for k in gem)
        g_n = max(sum(prof[k]["launches"] for k in gem), 1)
        kb = sum(prof[k]["bytes"] for k in gem) / g_n
        k_us = 1000 * g_ms / g_n
        kname = f"gemv_kernel ({g_n // 4} launches/step; {kind} peak)"
    achieved = kb / (k_us / 1e6) / 1e9 if k_us > 0 else 0.0
    if rank != 0:
        return 0
    traffic = STEP_KERNEL_DRAM_BYTES.get((args.model, world)) if m.kernels_per_step == 1 else None
    threads = host_threads()
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(path, args.cpu_steps, threads, cfg.vocab, 2)
    line = {
        "metric": "bs=1 decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_k/q6_k weights; u8 x s8 -> s32 tensor-core dots (exact), f32 scales and accumulation",
        "data": "synthetic (seeded random-init GGUF; uniform-random prompt ids)",
        "config": {"workload": f"{cfg.name} Q4_K_M bs=1 greedy decode",
                   "model": cfg.name, "global_batch": 1, "seq_len": PROMPT_LEN,
                   "context": f"{PROMPT_LEN + 1 + args.warmup}..{PROMPT_LEN + 1 + args.warmup + args.steps}",
                   "parallelism": f"tp{world}" if world > 1 else "single",
                   "l2": l2_note(wb, " per rank")},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": kname,
                     "bytes_per_launch": round(kb), "avg_launch_us": round(k_us, 3)},
        "step_roofline": {"weight_bytes_per_step_per_rank": wb, "achieved_gbs": round(step_gbs, 1),
                          "frac_of_peak": round(step_gbs / peak, 4)},
        # the separate-kernel path, timed kernel by kernel (serialised, for reference)
        "unfused_kernel_ms_per_step": {k: round(v["ms"] / 4, 4) for k, v in prof.items() if v["launches"]},
        "gpu_launches": m.kernels_per_step * args.steps,
        "clocks": clk,
        "load_s": round(t_load, 1),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))
    m.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def run_gemv_sweep(args):
    """Standalone dequant-GEMV sweep (the TinyLlama layer shapes and the Llama-2-7B
    M x K grid) at batch 1 (af_gemv_f32) and batch B > 1 (B vectors against
    one pass over the weights, af_gemv_batched_f32): one JSON
    line per shape and batch, device-timed with CUDA events; weight copies
    rotate so every launch streams from HBM (> L2)."""
    import torch
    from llm_core_b200 import _lib, gguf
    lib = _lib.load()
    peak, kind = peaks()
    shapes = [(2048, 2048), (256, 2048), (5632, 2048), (2048, 5632)]
    shapes += [(m, k) for m in (2048, 4096, 11008, 32000) for k in (2048, 4096, 11008)]
    if args.shapes:
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
    types = [gguf.GGML_Q4_K, gguf.GGML_Q6_K] if args.types == "both" else [int(args.types)]
    batches = [int(b) for b in args.batches.split(",")]
    rng = np.random.default_rng(0)
    for t in types:
        for (m, k), B in [(sh, b) for sh in shapes for b in batches]:
            gen = gguf.random_q4k if t == gguf.GGML_Q4_K else gguf.random_q6k
            host = gen(rng, m * k // 256).reshape(-1)
            nbytes = lib.af_weight_bytes(t, m, k)
            copies = max(1, int(np.ceil(300e6 / nbytes)))
            src = torch.from_numpy(host).cuda()
            ws = []
            for _ in range(copies):
                w = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
                assert lib.af_weight_pack(w.data_ptr(), src.data_ptr(), t, m, k, None) == 0
                ws.append(w)
            x = torch.randn(B, k, device="cuda")
            y = torch.empty(B, m, device="cuda")
            st = torch.cuda.current_stream().cuda_stream

            def launch(w):
                if B == 1:
                    return lib.af_gemv_f32(y.data_ptr(), w.data_ptr(), t, x.data_ptr(), m, k, st)
                return lib.af_gemv_batched_f32(y.data_ptr(), w.data_ptr(), t, x.data_ptr(), m, k, B, st)
            for i in range(3):
                assert launch(ws[i % copies]) == 0
            n = max(args.steps, copies)
            # the n launches replayed as one CUDA graph, so that the host's
            # launch rate does not bound the device time of small shapes
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                st = side.cuda_stream
                with torch.cuda.graph(g, stream=side):
                    for i in range(n):
                        launch(ws[i % copies])
            torch.cuda.synchronize()
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000 / n
            del g
            alg = m * k // 256 * (144 if t == gguf.GGML_Q4_K else 210) + 4 * B * (k + m)
            gbs = alg / (us * 1e-6) / 1e9
            print(json.dumps({"kernel": "gemv_kernel" if B == 1 else "bgemv_kernel",
                              "type": "Q4_K" if t == 12 else "Q6_K", "M": m, "K": k,
                              "batch": B, "us": round(us, 2), "bytes": alg, "GBps": round(gbs, 1),
                              "frac": round(gbs / peak, 4), "peak": f"{peak} ({kind})", "copies": copies}))
            del ws, src
            torch.cuda.empty_cache()
    return 0


def run_prefill_sweep(args):
    """Prefill dequant-GEMM (tcgen05) at the Llama-2-7B linear-layer shapes for
    a 512-token prompt: one JSON line per shape,
    device-timed with CUDA events (the per-call staging of X included).
    `tflops` counts the algorithmic 2·M·K·T."""
    import torch
    from llm_core_b200 import _lib, gguf
    lib = _lib.load()
    pj = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak = float(json.load(open(pj))["bf16_tflops"]) if os.path.exists(pj) else 1590.0
    kind = "measured" if os.path.exists(pj) else "fallback"
    T = 512
    shapes = [(12288, 4096), (4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]
    if args.shapes:
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
    rng = np.random.default_rng(0)
    t = gguf.GGML_Q4_K
    for (m, k) in shapes:
        host = gguf.random_q4k(rng, m * k // 256).reshape(-1)
        src = torch.from_numpy(host).cuda()
        w = torch.empty(lib.af_weight_bytes(t, m, k), dtype=torch.uint8, device="cuda")
        assert lib.af_weight_pack(w.data_ptr(), src.data_ptr(), t, m, k, None) == 0
        x = torch.randn(T, k, device="cuda")
        y = torch.empty(T, m, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        for _ in range(3):
            assert lib.af_prefill_gemm_f32(y.data_ptr(), w.data_ptr(), t, x.data_ptr(), m, k, T, st) == 0
        n = max(3, min(args.steps, 20))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            lib.af_prefill_gemm_f32(y.data_ptr(), w.data_ptr(), t, x.data_ptr(), m, k, T, st)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / n
        tf = 2.0 * m * k * T / (us * 1e-6) / 1e12
        print(json.dumps({"kernel": "prefill_gemm_kernel", "type": "Q4_K", "M": m, "K": k, "tokens": T,
                          "us": round(us, 1), "tflops": round(tf, 1),
                          "frac": round(tf / peak, 4), "peak": f"{peak} ({kind}, bf16 burst; f16 operands run at the same rate)"}))
        del w, src, x, y
        torch.cuda.empty_cache()
    if not args.shapes:
        run_prompt_pass(args, peak, kind)
    return 0


def run_prompt_pass(args, peak, kind):
    """The whole batched prompt pass of the 7B model (af_engine_prefill_batched:
    prefill GEMMs, row kernels, one causal-attention launch per layer, the
    last token through the decode step) on a 512-token prompt: time to first
    token, and the same prompt fed token by token for comparison.  Host wall
    clock around the synchronous calls, after one untimed pass each."""
    from llm_core_b200 import gguf
    from llm_core_b200.engine import LlamaCudaModel
    cfg = gguf.PRESETS[args.model]
    path = model_file(args.model, 0, None)
    m = LlamaCudaModel(path)
    rng = np.random.default_rng(7)
    T = 512
    prompt = [1] + rng.integers(0, cfg.vocab, T - 1).tolist()
    res = {}
    for batched in (True, False):
        m.prefill(prompt, 0, want_logits=False, batched=batched)
        t0 = time.perf_counter()
        m.prefill(prompt, 0, want_logits=False, batched=batched)
        res[batched] = time.perf_counter() - t0
    m.close()
    print(json.dumps({"kernel": "prompt pass (af_engine_prefill_batched)", "model": cfg.name, "tokens": T,
                      "ttft_ms": round(1000 * res[True], 2), "prefill_tok_s": round(T / res[True], 1),
                      "token_by_token_ms": round(1000 * res[False], 2),
                      "speedup_vs_token_by_token": round(res[False] / res[True], 2)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--prompt-len", type=int, default=PROMPT_LEN, help="prompt tokens before the timed decode")
    ap.add_argument("--cpu-steps", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemv-sweep", action="store_true", help="standalone GEMV sweep (not the headline line)")
    ap.add_argument("--prefill-sweep", action="store_true", help="prefill GEMM at the 7B shapes, 512 tokens")
    ap.add_argument("--shapes", default="", help="sweep shapes, e.g. 4096x4096,32000x4096")
    ap.add_argument("--types", default="both", help="12 (Q4_K), 14 (Q6_K) or both")
    ap.add_argument("--batches", default="1", help="GEMV sweep batch sizes, e.g. 1,4,16")
    args = ap.parse_args()
    set_prompt_len(args.prompt_len)
    if args.gemv_sweep:
        return run_gemv_sweep(args)
    if args.prefill_sweep:
        return run_prefill_sweep(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
