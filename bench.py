"""Decode-throughput benchmark of the B200 backend (metric: decode tok/s, Qwen3.5-style Q4_K_M).

Workload: the ~2B-class hybrid (config 3, 28 layers = 21 Gated-DeltaNet + 7 gated GQA, E=2048,
FFN 6144, vocab 151936, Q4_K_M with Q6_K head/embeddings), random-init N(0, 0.02) weights written as a
synthetic GGUF from a fixed seed, a 512-token seeded prompt, greedy decode at batch 1 per sequence.
A "step" is one greedy decode step of every sequence this rank owns (embedding lookup, 28 layers, LM
head, on-device argmax). Multi-GPU (torchrun): each rank owns its own independent sequences on its own
GPU (batch sharding, weak scaling, no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
PEAKS = ROOT / "MEASURED_PEAKS.json"
# DRAM bytes (read + write) per decode step of k_decode_persistent on this workload, from an ncu capture
# of a 4-step launch (profiles/k_decode_persistent_config3.md); a launch of n steps moves n times this.
TRAFFIC_PER_STEP = 1.2543e9
FALLBACK_HBM_GBS = 6650.0
METRIC = "decode tok/s at batch 1 & 64 (Qwen3.5-style Q4_K_M); GEMV HBM GB/s vs 8 TB/s"


def load_pkg():
    if "xjb200" in sys.modules:
        return sys.modules["xjb200"]
    spec = importlib.util.spec_from_file_location("xjb200", ROOT / "meta-work_b200" / "__init__.py",
                                                  submodule_search_locations=[str(ROOT / "meta-work_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["xjb200"] = mod
    spec.loader.exec_module(mod)
    return mod


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def hbm_peak():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class NvmlClocks:
    """NVML sampling (every ~2 ms, read-only queries) during the timed region: SM clock, max SM clock,
    throttle reasons; the same counters nvidia-smi reports, at a rate that covers a ~100 ms region."""

    NAMES = [("hw_slowdown", "nvmlClocksThrottleReasonHwSlowdown"),
             ("hw_thermal_slowdown", "nvmlClocksThrottleReasonHwThermalSlowdown"),
             ("sw_thermal_slowdown", "nvmlClocksThrottleReasonSwThermalSlowdown"),
             ("sw_power_cap", "nvmlClocksThrottleReasonSwPowerCap")]

    def __init__(self, gpu: int):
        import threading
        import pynvml as nv
        self.nv = nv
        nv.nvmlInit()
        h = None
        try:   # the CUDA device's own NVML handle (CUDA and NVML may number GPUs differently)
            import torch
            pr = torch.cuda.get_device_properties(gpu)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            h = nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            h = nv.nvmlDeviceGetHandleByIndex(gpu)
        self.h = h
        self.max = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        self.bits = [(n, getattr(nv, c, 0)) for n, c in self.NAMES]
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        self.samples, self.stopping = [], False

        def run():
            while not self.stopping:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), reasons(h)))
                time.sleep(0.002)
        self.t = threading.Thread(target=run, daemon=True)
        self.t.start()
        while not self.samples:
            time.sleep(0.001)

    def stop(self):
        self.stopping = True
        self.t.join()
        sm = [float(c) for c, _ in self.samples]
        reasons = sorted({n for _, r in self.samples for n, b in self.bits if b and (r & b)})
        self.nv.nvmlShutdown()
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.max), "reasons": reasons,
                "samples": len(sm), "source": "nvml"}


def clocks_sampler(gpu: int):
    try:
        return NvmlClocks(gpu)
    except Exception:
        return Clocks(gpu)


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    def __init__(self, gpu: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
            return
        # the sampler takes a moment to start: wait (up to 10 s) for its first row so that the samples
        # cover the timed region that follows
        t0 = time.time()
        while time.time() - t0 < 10 and self.p.poll() is None:
            self.f.flush()
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.05)
        self.skip = sum(1 for _ in open(self.f.name))

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        lines = self.f.read().strip().splitlines()[getattr(self, "skip", 0):]   # rows from the timed region on
        rows = [r.split(",") for r in lines if r.count(",") >= 8]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def step_bytes(cfg, pos: int, kv_bytes: int = 2) -> dict:
    """Algorithmic HBM bytes of one batch-1 decode step at KV length `pos` (weights of all layers and the
    head read once, KV cache read + one position written, GDN + conv state read + written)."""
    from xjb200 import synth
    E, FF, V, L = cfg.n_embd, cfg.n_ff, cfg.n_vocab, cfg.n_layer
    H, Hkv, D = cfg.n_head, cfg.n_head_kv, cfg.head_dim
    S, Hk, Hv = cfg.s_k, cfg.h_k, cfg.h_v
    DI, KD = Hv * S, Hk * S
    CD = 2 * KD + DI
    bpw = {synth.Q4_K: 144 / 256, synth.Q6_K: 210 / 256, synth.Q8_0: 34 / 32, synth.F32: 4}

    def more_bits(i):
        return i < L // 8 or i >= 7 * L // 8 or (i - L // 8) % 3 == 2

    w = 0.0
    n_full = 0
    for i in range(L):
        down_t = synth.Q6_K if (cfg.wtype == synth.Q4_K and more_bits(i)) else cfg.wtype
        w += (2 * E * FF) * bpw[cfg.wtype] + FF * E * bpw[down_t] + 2 * E * 4
        if (i + 1) % cfg.full_attn_interval:
            w += (E * CD + E * DI + 2 * E * Hv + DI * E) * bpw[cfg.wtype] + (CD * cfg.conv_k + 3 * Hv + S) * 4
        else:
            n_full += 1
            v_t = synth.Q6_K if (cfg.wtype == synth.Q4_K and more_bits(i)) else cfg.wtype
            w += (E * 2 * H * D + E * Hkv * D + H * D * E) * bpw[cfg.wtype] + E * Hkv * D * bpw[v_t] + 2 * D * 4
    io_t = synth.Q6_K if cfg.wtype == synth.Q4_K else cfg.wtype
    head = E * V * bpw[io_t] + E * 4 + E * bpw[io_t]
    kv = n_full * 2 * Hkv * D * kv_bytes * (pos + 1)
    n_rec = L - n_full
    state = n_rec * (2 * Hv * S * S * 4 + 2 * CD * (cfg.conv_k - 1) * 4)
    return {"weights": w + head, "kv": kv, "state": state, "total": w + head + kv + state}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU path (oracle/_ref, the reference's own core/*.c) on the host cores."""
    if rank != 0:
        return
    from xjb200 import synth
    sys.path.insert(0, str(ROOT))
    from oracle import ref
    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libxjref.so was not built"}))
        return
    cfg = synth.CONFIG3
    mdir = os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models_r0")          # the repo arm's rank-0 model
    path = synth.model_path(cfg, mdir)
    if not path.exists():
        # the model writer (libxj_synth.so) runs in a child process, so this arm's process maps only the
        # reference's library
        subprocess.run([sys.executable, "-c", "import bench; bench.load_pkg(); from xjb200 import synth; "
                        f"synth.cached_gguf(synth.CONFIG3, {str(mdir)!r})"], cwd=str(ROOT), check=True)
    m = ref.Model(path)
    threads = os.cpu_count() or 1
    ref.set_threads(threads)
    # the repo arm's operating point: its 512-token prompt (prefill untimed), then K timed decode steps
    n_prompt = args.prompt
    K = min(args.steps, 48)
    p = np.random.default_rng(1234).integers(0, cfg.n_vocab, n_prompt)
    _, _, _, times = m.greedy(p, K + 1, max_batch=64, n_ctx=n_prompt + K + 16)
    v = K / times[1]
    sample = (f"{cfg.name}: {n_prompt}-token prompt (prefill untimed, {times[0]:.1f} s), {K} greedy decode steps at "
              f"batch 1 at positions {n_prompt}..{n_prompt + K - 1}, {threads} threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": args.warmup, "ms_per_step": round(1e3 / v, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{cfg.name} greedy decode, batch 1 per GPU", "prompt": n_prompt, "batch": 1,
                   "same_config": True},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def cpu_baseline(K_cap=24):
    """Reference CPU path timed on this host on a bounded sample of the workload."""
    from xjb200 import synth
    sys.path.insert(0, str(ROOT))
    from oracle import ref
    if not ref.available():
        return None
    cfg = synth.CONFIG3
    m = ref.Model(synth.cached_gguf(cfg))
    threads = os.cpu_count() or 1
    ref.set_threads(threads)
    p = np.random.default_rng(1234).integers(0, cfg.n_vocab, 32)
    _, _, _, times = m.greedy(p, K_cap + 1, max_batch=8, n_ctx=2048)
    v = K_cap / times[1]
    return {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{cfg.name}: 32-token prompt, {K_cap} greedy decode steps at batch 1 at positions 32..{32 + K_cap - 1} "
                      f"(oracle/_ref, {threads} threads)"}


def run_gdn(xjcuda, peak, peak_kind):
    """Gated DeltaNet decode (config 2): one Gated DeltaNet step of 16 heads x 128x128 fp32 state per sequence
    at batch 1 and 64 (the batch kernel of batched decode), states rotated over >= 256 MiB so that L2
    cannot serve them. Bytes = state read + written."""
    out = {"workload": "config2 GDN decode, 16 heads, S=128, fp32 state", "unit": "GB/s"}
    for B in (1, 64):
        ms = xjcuda.gdn_time(128, 16, B, iters=50)
        nbytes = 2 * B * 16 * 128 * 128 * 4
        gbs = nbytes / (ms / 1e3) / 1e9
        out[f"b{B}"] = {"us": round(ms * 1e3, 2), "state_bytes": nbytes, "achieved": round(gbs, 1),
                        "frac": round(gbs / peak, 4)}
    # prefill: 4096 tokens through the chunked kernels vs the token-by-token kernel (16 heads, S = 128);
    # the first call loads the kernels' modules, the second is timed
    xjcuda.gdn_prefill_check(128, 16, 16, 256)
    d_out, d_state, ms_c, ms_s = xjcuda.gdn_prefill_check(128, 16, 16, 4096)
    out["prefill_4096"] = {"chunked_ms": round(ms_c, 3), "token_by_token_ms": round(ms_s, 3),
                           "chunked_tok_s": round(4096 / (ms_c / 1e3), 1), "max_rel_diff_out": d_out,
                           "max_rel_diff_state": d_state}
    out["peak"] = peak
    out["peak_kind"] = peak_kind
    return out


def run_prefill(xjcuda, model, n_prompt, chunks=(8, 64, 512)):
    """Prompt processing of one sequence (config 3, the bench's n_prompt-token prompt) on stages that take
    the prompt in chunks of 8 tokens (the decode bench's stage: wide mma.sync GEMVs, token-by-token GDN)
    and of 64 or 512 tokens (tcgen05 GEMMs in 64-token launches, the chunked tensor-core GDN). Device
    time of the prompt's first n_prompt - 1 tokens (the last one is the first decode step), second of
    two runs."""
    p = np.random.default_rng(1234).integers(0, model.n_vocab, n_prompt).astype(np.int32)
    out = {"prompt": n_prompt, "unit": "tok/s"}
    for mb in chunks:
        st = xjcuda.Stage(model, 0, model.n_layer, n_prompt + 16, mb)
        ms = None
        for _ in range(2):
            st.reset()
            _, _, ms = st.decode(p, 1)
        st.close()
        out[f"chunk_{mb}"] = {"ms": round(float(ms[0]), 3), "tok_s": round((n_prompt - 1) / (float(ms[0]) / 1e3), 1)}
    return out


GEMV_SHAPES = ((2048, 2048), (6144, 2048), (2048, 6144), (151936, 2048))   # rows N x columns K


def run_gemv(xjcuda, synth, peak, peak_kind, batches=(1, 4, 16), types=("q4_k", "q6_k", "q8_0"), shapes=GEMV_SHAPES):
    """Dequant-fused GEMV microbenchmark (config 1): y = W x for W in Q4_K / Q6_K / Q8_0 quantised from
    seeded N(0, 0.02), shapes N x K of GEMV_SHAPES (the last one the LM head), B = 1, 4, 16 tokens of fp32
    x. Each launch reads another of >= 256 MiB of distinct device copies of W, so L2 cannot serve the
    weights; ms = CUDA-event average per launch. Algorithmic bytes = N*K*bpw + B*K*4 + B*N*4."""
    import numpy as np
    bpw = {xjcuda.Q4_K: 144 / 256, xjcuda.Q6_K: 210 / 256, xjcuda.Q8_0: 34 / 32}
    names = {xjcuda.Q4_K: "q4_k", xjcuda.Q6_K: "q6_k", xjcuda.Q8_0: "q8_0"}
    rng = np.random.default_rng(11)
    pool = (rng.standard_normal(max(n * k for n, k in shapes), dtype=np.float32) * 0.02)
    out = {"workload": "config1 GEMV, weights rotated over >= 256 MiB of copies", "unit": "GB/s",
           "peak": peak, "peak_kind": peak_kind}
    best = None
    for t in (xjcuda.Q4_K, xjcuda.Q6_K, xjcuda.Q8_0):
        if names[t] not in types:
            continue
        for n, k in shapes:
            raw = synth.quantize_row(t, pool[:n * k])
            wbytes = len(raw)
            copies = max(2, -(-(256 << 20) // wbytes))
            for B in batches:
                ms = xjcuda.gemv_time(t, raw, k, n, T=B, copies=copies, iters=40)
                nbytes = n * k * bpw[t] + B * k * 4 + B * n * 4
                gbs = nbytes / (ms / 1e3) / 1e9
                key = f"{names[t]}_{n}x{k}_b{B}"
                out[key] = {"us": round(ms * 1e3, 2), "achieved": round(gbs, 1), "frac": round(gbs / peak, 4)}
                if best is None or gbs > best[1]:
                    best = (key, gbs)
    out["best"] = {"case": best[0], "frac": round(best[1] / peak, 4)}
    return out


def gemv_kw(args) -> dict:
    return {"types": tuple(args.gemv_types.split(",")),
            "shapes": GEMV_SHAPES if args.gemv_shapes == "all" else GEMV_SHAPES[-1:],
            "batches": tuple(int(b) for b in args.gemv_batches.split(","))}


def run_spec(args, model, rank, world, barrier, xjcuda, synth, local):
    """Speculative decoding (config 4): target = config 3, draft = the E=1024 8-layer Q8_0 model with the
    target's vocabulary, k = 4, greedy acceptance; args.spec seeded 256-token prompts in total, sharded
    over the ranks (args.spec / world sequences per GPU), args.spec_gen tokens each. Every GPU decodes its
    sequences as one batch (xj_cuda_batch_spec_decode): the draft proposes k tokens per sequence, the
    target verifies k + 1 tokens of all its sequences in one forward on the tensor cores. Output ids equal
    plain greedy decoding (tested). Timed: the whole call (prompts included), device time on the target's
    stream, max over ranks; e2e = the same call by the host clock."""
    import torch
    dpath = synth.cached_gguf(synth.DRAFT, os.environ.get("XJ_MODEL_DIR", f"/tmp/xj_models_r{local}"))
    dmodel = xjcuda.Model(dpath)
    n_prompt, n_gen, k = 256, args.spec_gen, 4
    per = max(1, args.spec // world)
    allp = np.random.default_rng(777).integers(0, model.n_vocab, (per * world, n_prompt)).astype(np.int32)
    prompts = allp[rank * per:(rank + 1) * per]
    n_ctx = n_prompt + n_gen * (k + 1) + k + 8
    target = xjcuda.Batch(model, per, n_ctx, max_tokens=k + 1)
    draft = xjcuda.Batch(dmodel, per, n_ctx, max_tokens=8)
    barrier()
    t0 = time.perf_counter()
    _, st, ms = target.spec_decode(draft, prompts, n_gen, k)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3
    target.close()
    draft.close()
    v = torch.tensor([ms, wall, st[0]], device="cuda", dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
    t_max, w_max, rounds_max = float(v[0]), float(v[1]), int(v[2])
    if rank != 0:
        return None
    total = per * world
    return {"workload": "config4 speculative: target config3, draft 1024x8 Q8_0 (vocab 151936), k=4, batched verify",
            "sequences_total": total, "sequences_per_gpu": per, "prompt": n_prompt, "gen": n_gen,
            "value": round(total * n_gen / (t_max / 1e3), 1), "unit": "emitted tok/s",
            "accepted_tok_s_rank0": round(st[2] / (t_max / 1e3), 1),
            "target_forwards_per_s": round(rounds_max / (t_max / 1e3), 2),
            "target_rows_per_s": round(world * st[3] * per / (t_max / 1e3), 1),
            "acceptance": round(st[2] / max(1, st[1]), 4),
            "rounds_rank0": st[0], "drafted_rank0": st[1], "accepted_rank0": st[2],
            "e2e": {"value": round(total * n_gen / (w_max / 1e3), 1), "unit": "emitted tok/s", "step": "one verify round",
                    "h2d_bytes_per_step": round(4 * per * n_prompt / max(1, st[0]), 1),
                    "d2h_bytes_per_step": round(4 * per + 4 * per * n_gen / max(1, st[0]), 1)},
            "timing": "device time of one xj_cuda_batch_spec_decode call per GPU (prompts included), max over ranks"}


def run_batch(args, cfg, model, rank, world, barrier, xjcuda, n_seq=None):
    """Batched greedy decode: args.batch (or n_seq) independent sequences per GPU in lockstep
    (xj_cuda_batch_*), each with its own seeded prompt of args.prompt tokens; K timed steps = one token of
    every sequence."""
    import torch
    B = n_seq or args.batch
    n_ctx = args.prompt + max(args.warmup, 3) + 2 * args.steps + 16
    bt = xjcuda.Batch(model, B, n_ctx, max_tokens=16)                # prompts in chunks of 16 tokens per sequence
    P = np.random.default_rng(4321 + rank).integers(0, cfg.n_vocab, (B, args.prompt)).astype(np.int32)
    toks, _, ms_pre = bt.decode(P, max(args.warmup, 3))          # prompt + warm-up steps (untimed)
    last = toks[:, -1:]
    pos0 = bt.n_past
    barrier()
    toks, _, ms = bt.decode(last, args.steps)
    barrier()
    dev_ms = float(ms[0] + ms[1])
    launches = bt.last_launches()
    last = toks[:, -1:]
    barrier()
    t0 = time.perf_counter()
    bt.decode(last, args.steps)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3
    t_max, e2e_max = dev_ms, e2e_ms
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dev_ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max, e2e_max = float(t[0]), float(t[1])
    bt.close()
    if rank != 0:
        return None
    b = step_bytes(cfg, pos0 + args.steps // 2)
    step_total = b["weights"] + B * (b["kv"] + b["state"])
    peak, peak_kind = hbm_peak()
    achieved = step_total / (t_max / args.steps / 1e3) / 1e9
    return {
        "value": round(world * B * args.steps / (t_max / 1e3), 1), "unit": "tok/s", "sequences_per_gpu": B,
        "ms_per_step": round(t_max / args.steps, 4), "steps": args.steps, "prompt": args.prompt,
        "e2e": {"value": round(world * B * args.steps / (e2e_max / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": round(4 * B / args.steps, 3), "d2h_bytes_per_step": 4 * B},
        "roofline": {"bound": "hbm", "kernel": "decode-step CUDA graph (batched)", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "bytes_per_step": round(step_total), "peak_kind": peak_kind},
        # the north-star wording: weight + KV bytes per token over the nominal 8 TB/s (roofline.frac above
        # also counts the recurrent state and uses the measured copy bandwidth)
        "baseline_roofline": {"bytes_per_token": round((b["weights"] + B * b["kv"]) / B),
                              "frac_of_8tbs": round((b["weights"] + B * b["kv"]) / (t_max / args.steps / 1e3) / 8e12, 4)},
        "gpu_launches": int(sum(launches)), "prompt_ms": round(float(ms_pre[0]), 1),
    }


def run_pipeline_native(args, cfg, model, rank, world, barrier, xjcuda):
    """Layer pipeline over all ranks, native (xj_cuda_pipeline_*: NCCL send/recv of activations and ids
    inside libxj_cuda.so): args.batch sequences in total, args.micro_batches micro-batches, rank r holding
    an even share of the layers. The communicator identifier goes from rank 0 to the others through
    torch.distributed (this harness's channel). Timed: K decode steps in one decode call, device time per
    rank (CUDA events on its compute stream), max over ranks; e2e = the same call by the host clock (prompt
    upload and id download included)."""
    import torch
    import torch.distributed as dist
    t = torch.zeros(xjcuda.PIPELINE_ID_BYTES, dtype=torch.uint8, device="cuda")
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(xjcuda.pipeline_id()), dtype=torch.uint8))
    dist.broadcast(t, 0)
    pid = bytes(t.cpu().numpy().tobytes())
    B = args.batch
    n_ctx = args.prompt + max(args.warmup, 3) + 2 * args.steps + 16
    p = xjcuda.Pipeline(model, rank, world, pid, B, n_ctx, args.micro_batches)
    prompts = np.random.default_rng(4321).integers(0, cfg.n_vocab, (B, args.prompt)).astype(np.int32)
    out, ms_pre = p.decode(prompts if rank == 0 else args.prompt, max(args.warmup, 3))   # prompt + warm-up
    last = out[:, -1:] if rank == 0 else 1
    barrier()
    out, ms = p.decode(last, args.steps)
    barrier()
    last = out[:, -1:] if rank == 0 else 1
    t0 = time.perf_counter()
    p.decode(last, args.steps)
    e2e_ms = (time.perf_counter() - t0) * 1e3
    barrier()
    v = torch.tensor([ms, e2e_ms], device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    t_max, e2e_max = float(v[0]), float(v[1])
    p.close()
    if rank != 0:
        return None
    L = model.n_layer
    return {
        "value": round(B * args.steps / (t_max / 1e3), 1), "unit": "tok/s", "scaling": "strong",
        "sequences_total": B, "micro_batches": args.micro_batches, "ms_per_step": round(t_max / args.steps, 4),
        "steps": args.steps, "prompt": args.prompt, "prompt_ms": round(ms_pre, 1),
        "layers_per_rank": [L // world + (1 if r < L % world else 0) for r in range(world)],
        "e2e": {"value": round(B * args.steps / (e2e_max / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": round(4 * B / args.steps, 3), "d2h_bytes_per_step": 4 * B},
        "exchange_bytes_per_step": {"activations": int(B * cfg.n_embd * 4 * (world - 1)), "ids": 4 * B},
        "transport": "NCCL send/recv inside libxj_cuda.so",
    }


def run_pipeline(args, rank, local, world):
    """--pipeline: only the native layer pipeline over the ranks (run_pipeline_native), as its own line."""
    import datetime
    import torch
    import torch.distributed as dist
    from xjb200 import synth, xjcuda
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = synth.CONFIG3
    model = xjcuda.Model(synth.cached_gguf(cfg, os.environ.get("XJ_MODEL_DIR", f"/tmp/xj_models_r{local}")))

    def barrier():
        torch.cuda.synchronize()
        dist.barrier()

    line = run_pipeline_native(args, cfg, model, rank, world, barrier, xjcuda)
    if rank == 0:
        print(json.dumps({"metric": "pipelined batched decode tok/s (config 3, Q4_K_M)", "n_gpus": world,
                          "higher_is_better": True, "data": "synthetic", "vs_baseline": None,
                          "config": {"workload": f"{cfg.name} greedy decode, {args.batch} sequences",
                                     "parallelism": f"layer pipeline x{world}"}, **line}))
    dist.destroy_process_group()


def run_phase_trace(args) -> dict:
    """Per-phase timing of the persistent decode kernel (XJC_OPT_TRACE) on config 3 after the
    --prompt-token prompt: the last of 8 traced steps, summed per phase kind and per slot of a layer
    (in-projection, GDN / attention, out-projection, FFN gate + up, FFN down), plus the attention items'
    steps. Times are us on the device clock."""
    from xjb200 import synth, xjcuda
    cfg = synth.CONFIG3
    model = xjcuda.Model(synth.cached_gguf(cfg, os.environ.get("XJ_MODEL_DIR", "/tmp/xj_models_r0")))
    stage = xjcuda.Stage(model, 0, model.n_layer, args.prompt + 64, 8)
    prompt = np.random.default_rng(1234).integers(0, cfg.n_vocab, args.prompt).astype(np.int32)
    toks, _, _ = stage.decode(prompt, 4)
    toks, _, _ = stage.decode(toks[-1:], 20)
    xjcuda.set_option(xjcuda.OPT_TRACE, 1)
    try:
        _, _, ms = stage.decode(toks[-1:], 8)
        t = stage.phase_trace()
    finally:
        xjcuda.set_option(xjcuda.OPT_TRACE, 0)
        stage.close()
    kinds = {0: "gemv", 1: "gdn", 2: "attn", 3: "argmax"}
    ends = t[:, 4] + t[:, 3]
    out = {"prompt": args.prompt, "ms_per_traced_step": round(float(ms[1]) / 8, 4), "phases": int(len(t)),
           "step_span_us": round(float(ends[-1] - t[0, 4]), 1),
           "barrier_gaps_us": round(float((t[1:, 4] - ends[:-1]).sum()), 1)}
    nl = model.n_layer
    slots = ["in_proj", "mixer", "out_proj", "ffn_gate_up", "ffn_down"]
    for k, name in enumerate(slots):
        sel = t[k:5 * nl:5]
        out[name] = {"max_cta_us": round(float(sel[:, 1].sum()), 1), "span_us": round(float(sel[:, 3].sum()), 1)}
        if k != 1:
            out[name]["prologue_us"] = round(float(sel[:, 7].sum()), 1)
    out["lm_head_span_us"] = round(float(t[5 * nl:-1, 3].sum()), 1)
    at = t[t[:, 0] == 2]
    if len(at):
        out["attention_item_us"] = {k: round(float(at[:, i].mean()), 2) for k, i in
                                    (("to_item", 7), ("qk_norm_rope", 8), ("rows", 9), ("rounds", 10),
                                     ("split_counter", 11), ("merge", 12), ("phase_max", 1))}
    out["by_kind_max_cta_us"] = {kinds.get(k, str(k)): round(float(t[t[:, 0] == k, 1].sum()), 1) for k in kinds}
    out["phases_by_kind"] = {kinds.get(k, str(k)): int((t[:, 0] == k).sum()) for k in kinds}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemv", type=int, default=1, help="run the config-1 GEMV microbenchmark on rank 0 (0: skip)")
    ap.add_argument("--only", choices=["gemv", "trace", "gdn", "prefill"], default=None,
                    help="run only this microbenchmark (one GPU; e.g. under a profiler) and print its JSON")
    ap.add_argument("--prefill-chunks", default="8,64,512", help="prompt chunk sizes (stage max_batch) of the prefill leg")
    ap.add_argument("--gemv-types", default="q4_k,q6_k,q8_0")
    ap.add_argument("--gemv-shapes", default="all", help="'all' or 'lm' (the 151936 x 2048 LM head only)")
    ap.add_argument("--gemv-batches", default="1,4,16")
    ap.add_argument("--batch", type=int, default=64, help="sequences of the batched-decode measurement (0: skip)")
    ap.add_argument("--pipeline", action="store_true",
                    help="under torchrun: one layer range per GPU (NCCL layer pipeline) on --batch sequences")
    ap.add_argument("--micro-batches", type=int, default=2)
    ap.add_argument("--strong", type=int, default=1,
                    help="with several GPUs, also time --batch sequences in total: sharded and through the layer pipeline")
    ap.add_argument("--spec", type=int, default=64,
                    help="config 4: batched speculative decoding of this many 256-token prompts in total (0: skip)")
    ap.add_argument("--spec-gen", type=int, default=256, help="config 4: tokens generated per prompt")
    args = ap.parse_args()
    rank, local, world = dist_env()
    load_pkg()
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    torch.cuda.set_device(local)
    if args.pipeline:
        return run_pipeline(args, rank, local, world)
    if args.only == "gemv":
        from xjb200 import synth, xjcuda
        peak, peak_kind = hbm_peak()
        print(json.dumps({"gemv": run_gemv(xjcuda, synth, peak, peak_kind, **gemv_kw(args))}))
        return
    if args.only == "trace":
        print(json.dumps({"phase_trace": run_phase_trace(args)}))
        return
    if args.only == "prefill":
        from xjb200 import synth, xjcuda
        model = xjcuda.Model(synth.cached_gguf(synth.CONFIG3, os.environ.get("XJ_MODEL_DIR", f"/tmp/xj_models_r{local}")))
        chunks = tuple(int(c) for c in args.prefill_chunks.split(","))
        print(json.dumps({"prefill": run_prefill(xjcuda, model, args.prompt, chunks)}))
        return
    if args.only == "gdn":
        from xjb200 import xjcuda
        peak, peak_kind = hbm_peak()
        print(json.dumps({"gdn": run_gdn(xjcuda, peak, peak_kind)}))
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from xjb200 import synth, xjcuda
    cfg = synth.CONFIG3
    path = synth.cached_gguf(cfg, os.environ.get("XJ_MODEL_DIR", f"/tmp/xj_models_r{local}"))
    model = xjcuda.Model(path)
    n_vt = min(args.steps, 32)                                        # steps of the vtable e2e run
    n_ctx = args.prompt + max(args.warmup, 3) + 3 * args.steps + n_vt + 16   # prefill + warm-up + timed, e2e, sampled runs
    stage = xjcuda.Stage(model, 0, model.n_layer, n_ctx, 8)
    prompt = np.random.default_rng(1234 + rank).integers(0, cfg.n_vocab, args.prompt).astype(np.int32)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # prefill + warm-up decode steps (untimed)
    toks, _, _ = stage.decode(prompt, max(args.warmup, 3))
    last = toks[-1:]
    pos0 = stage.n_past
    # timed region: exactly K decode steps, device-timed with CUDA events on the stage stream
    barrier()
    clocks = clocks_sampler(local)
    toks, _, ms = stage.decode(last, args.steps)
    barrier()
    clk = clocks.stop()
    dev_ms = float(ms[0] + ms[1])
    kern_ms = float(ms[1])                     # the persistent launch: all K steps (one launch)
    launches = stage.last_decode_launches()
    last = toks[-1:]
    # end to end through the public C ABI with host buffers (token ids in, ids out), host wall clock
    barrier()
    t0 = time.perf_counter()
    toks2, _, _ = stage.decode(last, args.steps)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3
    # end to end through the drop-in vtable with host buffers, as the runtime's pipeline drives a stage
    # (core/xj_net.c:532-605 via xj_pipeline_eval): embed on the host (xjc_embed), forward [1][E] in,
    # logits [1][V] out, argmax on the host; n_vt steps by the host clock
    tok = int(toks2[-1])
    barrier()
    t0 = time.perf_counter()
    for _ in range(n_vt):
        x = stage.forward(model.embed_many([tok]))
        tok = int(np.argmax(stage.logits(x)[0]))
    vt_ms = (time.perf_counter() - t0) * 1e3
    # sampled decode (top-40 / top-p 0.95 / temperature 0.9, the session's settings) on the device: the
    # same persistent kernel with its SAMPLE phase; device time of args.steps steps
    stage.set_sampler(0.9, 1234 + rank)
    stoks, _, sms = stage.decode(np.array([tok], np.int32), args.steps)
    samp_launches = stage.last_decode_launches()[1]
    stage.set_sampler(0.0)
    samp_ms = float(sms[0] + sms[1])
    t_max = dev_ms
    e2e_max = e2e_ms
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dev_ms, e2e_ms, vt_ms, samp_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_max, e2e_max, vt_ms, samp_ms = float(t[0]), float(t[1]), float(t[2]), float(t[3])
    value = world * args.steps / (t_max / 1e3)
    e2e = world * args.steps / (e2e_max / 1e3)
    stage.close()
    batch_line = run_batch(args, cfg, model, rank, world, barrier, xjcuda) if args.batch > 0 else None
    # strong scaling: args.batch sequences in total over the ranks (batch sharding, no data-path
    # collective), and the same total through the layer pipeline over all ranks
    strong_line = None
    pipe_line = None
    if world > 1 and args.batch > 0 and args.strong:
        strong_line = run_batch(args, cfg, model, rank, world, barrier, xjcuda, n_seq=max(1, args.batch // world))
        if strong_line:
            strong_line["scaling"] = "strong"
            strong_line["sequences_total"] = max(1, args.batch // world) * world
        pipe_line = run_pipeline_native(args, cfg, model, rank, world, barrier, xjcuda)
    spec_line = run_spec(args, model, rank, world, barrier, xjcuda, synth, local) if args.spec > 0 else None
    if rank == 0:
        peak, peak_kind = hbm_peak()
        b = step_bytes(cfg, pos0 + args.steps // 2)
        persistent = launches[1] == 1
        n_kern = args.steps if persistent else args.steps - 1   # the persistent launch runs every step
        achieved = b["total"] * n_kern / (kern_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_k/q6_k weights, f32 accumulate", "data": "synthetic",
            "config": {"workload": f"{cfg.name} greedy decode, batch 1 per GPU", "prompt": args.prompt,
                       "batch_per_gpu": 1, "kv_cache": "f16", "parallelism": f"batch-shard x{world}",
                       "decode_kernel": "persistent" if launches[1] == 1 else "graph",
                       "l2": "weights 1.2 GB per step > 126 MB L2"},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": round(4 / args.steps, 3),
                    "d2h_bytes_per_step": 4},
            "e2e_vtable": {"value": round(world * n_vt / (vt_ms / 1e3), 2), "unit": "tok/s", "steps": n_vt,
                           "h2d_bytes_per_step": 4 * cfg.n_embd, "d2h_bytes_per_step": 4 * cfg.n_vocab + 4 * cfg.n_embd,
                           "path": "xj_stage forward + logits with host buffers, argmax and embedding on the host"},
            "sampled": {"value": round(world * args.steps / (samp_ms / 1e3), 2), "unit": "tok/s",
                        "sampler": "temperature 0.9, top-k 40, top-p 0.95, seeded per position",
                        "decode_kernel": "persistent" if samp_launches == 1 else "graph",
                        "timing": "device time of one xj_cuda_decode call, max over ranks"},
            "roofline": {"bound": "hbm",
                         "kernel": "k_decode_persistent" if persistent else "decode-step CUDA graph",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": round(TRAFFIC_PER_STEP * n_kern) if persistent else None,
                         "algorithmic_bytes": round(b["total"] * n_kern), "units": f"{n_kern} decode steps",
                         "launch_ms": round(kern_ms, 4), "peak_kind": peak_kind},
            # the north-star wording: weight + KV bytes per token over the nominal 8 TB/s (roofline.frac
            # also counts the recurrent state and uses the measured copy bandwidth)
            "baseline_roofline": {"bytes_per_token": round(b["weights"] + b["kv"]),
                                  "frac_of_8tbs": round((b["weights"] + b["kv"]) * args.steps / (t_max / 1e3) / 8e12, 4)},
            "clocks": clk,
            "gpu_launches": int(sum(launches)),
            "tokens_check": int(toks[0]),
        }
        if batch_line:
            line["batch"] = batch_line
        if strong_line:
            line["strong"] = strong_line
        if pipe_line:
            line["pipeline"] = pipe_line
        line["gdn"] = run_gdn(xjcuda, peak, peak_kind)
        line["prefill"] = run_prefill(xjcuda, model, args.prompt, tuple(int(c) for c in args.prefill_chunks.split(",")))
        # the same GDN step inside the persistent decode kernel (config 3 has 21 such layers of 16 heads x
        # 128x128): mean over its GDN phases of the slowest CTA, from a short traced decode
        tr = run_phase_trace(args)
        n_gdn = tr["phases_by_kind"]["gdn"]
        if n_gdn:
            us = tr["by_kind_max_cta_us"]["gdn"] / n_gdn
            nbytes = 2 * 16 * 128 * 128 * 4
            line["gdn"]["b1_in_persistent_kernel"] = {
                "us": round(us, 2), "state_bytes": nbytes, "achieved": round(nbytes / (us / 1e6) / 1e9, 1),
                "frac": round(nbytes / (us / 1e6) / 1e9 / peak, 4),
                "timing": "phase trace (device clock), slowest CTA of each GDN phase, mean over the step's 21 layers"}
        if args.gemv:
            line["gemv"] = run_gemv(xjcuda, synth, peak, peak_kind, **gemv_kw(args))
        if spec_line:
            line["spec"] = spec_line
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
