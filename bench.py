"""Benchmark of the speculative-decoding step (MTP draft -> verify forward ->
acceptance -> KV commit/rollback) on B200.

Default workload: Llama-3-8B-shape W4A16 chain speculative decoding, batch 32
sequences per GPU, 2048-token contexts, draft length 4 (3 MTP heads),
temperature 0.8, seed 1.  Weights are synthetic int4 (group 128, fp16 scales,
N(0, 0.02) draws); the KV cache is seeded with random fp16 values (no prefill
in the timed setup).  Sequences are sharded by request: every rank holds a
full weight replica and its own sequences (weak scaling, no collective on
the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 8b|tree|14b|tiny]
    python bench.py --impl reference ...   # CPU restatement on the host cores
    python bench.py --kernel gemm --shape 160,128256,4096   # one hot kernel (profiling)
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
sys.path.insert(0, os.path.join(ROOT, "sme-llm-edge_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CONFIGS = {
    "8b": dict(shape="llama3-8b", batch=32, ctx=2048, draft_len=4, temperature=0.8, seed=1, tree=None),
    "tree": dict(shape="llama3-8b", batch=16, ctx=4096, draft_len=0, temperature=1.0, seed=2, tree=[4, 4, 2, 2]),
    "14b": dict(shape="14b", batch=64, ctx=8192, draft_len=4, temperature=0.8, seed=3, tree=None, ragged=(1024, 8192)),
    "tiny": dict(shape="tiny", batch=1, ctx=512, draft_len=3, temperature=1.0, seed=0, tree=None),
}
METRIC = "accepted tokens/s, 8B-shape W4A16 MTP spec-decode, 1/2/4/8 B200; verify µs"
# DRAM bytes read + written by one launch, from the ncu captures summarised
# under profiles/: (traffic, launch, algorithmic bytes of that launch)
TRAFFIC = {
    "lm_head": (332.8e6, "lm_head M=160 N=128256 K=4096", 271.3e6),
    "attention": (275.5e6, "attention B=32 R=5 Hq=32 Hkv=8 hd=128 ctx=2048", 269.1e6),
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML polled every ~2 ms from a thread (the timed steps are tens of
    ms), the device matched by PCI bus id; nvidia-smi -lms 200 as a fallback.
    Read-only: no clock or power setting is touched."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.nv = None
        self.samples = []
        self.stop_flag = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.index)
            bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        try:
            self.nv, self.h = self._nvml_handle()
            self.max_mhz = float(self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _poll(self):
        nv, h = self.nv, self.h
        while not self.stop_flag.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                bits = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((mhz, bits))
            except Exception:
                pass
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        self.stop_flag.set()
        if self.nv is not None:
            self.t.join(timeout=5)
            sm = [m for m, _ in self.samples]
            reasons = sorted({n for _, bits in self.samples for n, bit in self.REASONS if bits & bit})
            return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": self.max_mhz,
                    "sm_min_mhz": min(sm) if sm else None, "reasons": reasons, "samples": len(sm),
                    "source": "nvml, every ~2 ms during the timed steps"}
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi -lms 200"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def reduce_max(pg, x: float, local: int) -> float:
    from specdec.dist import reduce_max as rmax

    return rmax(pg, x, f"cuda:{local}")


def reduce_sum(pg, x: float, local: int) -> float:
    from specdec.dist import reduce_sum as rsum

    return rsum(pg, x, f"cuda:{local}")


def barrier(pg, local):
    if pg is not None:
        import torch

        pg.barrier(device_ids=[local])
        torch.cuda.synchronize()


def ctx_lengths(cfg, rank, world=1):
    """Context lengths of this rank's sequences: the global batch (batch per
    GPU x world) is drawn once and sharded by request."""
    from specdec.dist import shard_range

    B = cfg["batch"]
    if cfg.get("ragged"):
        lo, hi = cfg["ragged"]
        rng = np.random.default_rng(cfg["seed"] * 1000)
        glob = rng.integers(lo, hi + 1, B * world).astype(np.int32)
    else:
        glob = np.full(B * world, cfg["ctx"], np.int32)
    a, b = shard_range(B * world, world, rank)
    return glob[a:b]


def workload_bytes_flops(shape, ctx, rows, weight_bytes):
    """Algorithmic bytes of one verify step: W4 weights + scales of all layers and
    lm_head read once, fp16 K/V of every context token of every sequence read once."""
    kv_per_tok = shape["layers"] * shape["n_kv_heads"] * shape["head_dim"] * 2 * 2
    kv_bytes = float(np.sum(ctx.astype(np.float64) + rows)) * kv_per_tok
    H, F, V, L = shape["hidden"], shape["ffn"], shape["vocab"], shape["layers"]
    qd, kd = shape["n_q_heads"] * shape["head_dim"], shape["n_kv_heads"] * shape["head_dim"]
    params = L * (H * (qd + 2 * kd) + qd * H + 2 * H * F + F * H) + H * V
    return weight_bytes + kv_bytes, kv_bytes, 2.0 * params


# ------------------------------------------------------------ CPU baseline
# The oracle port (C, OpenMP) on the host cores: the same batched step as the
# GPU arm -- MTP draft chain, verify forward over the paged KV, acceptance --
# timed on a sample of CPU_SAMPLE_SEQS of the batch's sequences per step.  The
# CPU's work is linear in the sequences (no weight reuse across rows in the
# oracle's contraction), so tokens / time of the sample is the batch's rate.
CPU_SAMPLE_SEQS = 4


def _model_shape(cfg):
    from model_shapes import MODEL_SHAPES  # pure Python: loads no library

    return MODEL_SHAPES[cfg["shape"]]


def cpu_setup(cfg, rng):
    """A 1-decoder-layer oracle model of the config and a paged KV of the
    sample's sequences (weights synthesised, KV filled at random; not timed).
    The other layers are identical in cost: their time is the per-layer time
    measured here as the forward with one layer minus the forward with none."""
    import oracle as O

    shape = _model_shape(cfg)
    t0 = time.time()
    ocfg = dict(shape, layers=1, block_size=16, rms_eps=1e-5, rope_theta=10000.0)
    m = O.OracleModel(ocfg, seed=cfg["seed"], rope_max_pos=int(cfg["ctx"]) + 80)
    k = cfg["draft_len"] or 4
    R, ctx, n = k + 1, int(cfg["ctx"]), min(CPU_SAMPLE_SEQS, cfg["batch"])
    mbpr = (ctx + R + 15) // 16 + 1
    kv = O.OracleKV(1, n * mbpr, shape["n_kv_heads"], 16, shape["head_dim"])
    kv.pool[:] = O.f16_bits(rng.uniform(-1, 1, kv.pool.shape).astype(np.float32))
    st = dict(model=m, kv=kv, n=n, k=k, R=R, ctx=ctx, shape=shape,
              tables=np.arange(n * mbpr, dtype=np.int32).reshape(n, mbpr),
              ctxs=np.full(n, ctx, np.int32),
              pos=np.tile(np.arange(ctx, ctx + R, dtype=np.int32), n),
              mask=np.array([(1 << (r + 1)) - 1 for r in range(R)], np.uint64),
              setup_s=time.time() - t0)
    toks = rng.integers(0, shape["vocab"], n * R).astype(np.int32)
    t = []
    for nl in (0, 1):
        t1 = time.time()
        O.forward(m, kv, st["tables"], st["ctxs"], toks, st["pos"], st["pos"], st["mask"], n, R, n_layers=nl,
                  want_hidden=False)
        t.append(time.time() - t1)
    st["t_layer"] = max(0.0, t[1] - t[0])
    return st


def cpu_sample(cfg, st, rng, step):
    """One timed sample: the batched step of st['n'] sequences on the 1-layer
    model, plus (layers - 1) x the per-layer time.  Returns (tokens, seconds)."""
    import oracle as O

    shape, n, k, R = st["shape"], st["n"], st["k"], st["R"]
    H, V = shape["hidden"], shape["vocab"]
    h0 = rng.standard_normal((n, H)).astype(np.float32)
    pend = rng.integers(0, V, n).astype(np.int32)
    T = cfg["temperature"]
    t1 = time.time()
    dl, drafts, _ = O.draft_chain(st["model"], h0, k, T, 1.0, cfg["seed"], step)
    toks = np.concatenate([pend[:, None], drafts], axis=1).reshape(-1).astype(np.int32)
    lg, _ = O.forward(st["model"], st["kv"], st["tables"], st["ctxs"], toks, st["pos"], st["pos"], st["mask"], n, R,
                      want_hidden=False)
    acc, _ = O.accept_chain(lg.reshape(n, R, V), dl, drafts, T, 1.0, cfg["seed"], step)
    secs = (time.time() - t1) + (shape["layers"] - 1) * st["t_layer"]
    return int(np.sum(acc + 1)), secs


def cpu_describe(cfg, st, samples):
    shape = st["shape"]
    return (f"{samples} sample(s) of {st['n']} of the batch's {cfg['batch']} sequences ({st['n'] * st['R']} verify "
            f"rows, ctx {st['ctx']}, chain {st['k']}, T {cfg['temperature']}): MTP draft chain, verify forward and "
            f"acceptance on a 1-decoder-layer copy, timed, plus {shape['layers'] - 1} layers x "
            f"{st['t_layer']:.3f} s (forward with one layer minus forward with none, measured once); rate = "
            f"sum(accepted + 1) / time, linear in the sequences; OpenMP threads = {os.cpu_count()}; "
            f"x86-64 scalar/auto-vectorised C, ARM SVE2/SME unavailable; weight synthesis {st['setup_s']:.1f}s "
            f"not timed")


def cpu_baseline(cfg, samples=2):
    rng = np.random.default_rng(7)
    st = cpu_setup(cfg, rng)
    try:
        tok = secs = 0.0
        for i in range(samples):
            a, b = cpu_sample(cfg, st, rng, i)
            tok, secs = tok + a, secs + b
        return {"value": tok / secs, "unit": "accepted tokens/s", "cores": os.cpu_count(), "kind": "port",
                "sample": cpu_describe(cfg, st, samples)}
    finally:
        st["model"].close()


def run_reference(args, world, rank):
    if rank != 0:
        return
    cfg = dict(CONFIGS[args.config])
    rng = np.random.default_rng(7)
    st = cpu_setup(cfg, rng)  # once; each step below times one sample of the batched step
    tok = secs = 0.0
    try:
        for i in range(args.warmup + args.steps):
            a, b = cpu_sample(cfg, st, rng, i)
            if i >= args.warmup:
                tok, secs = tok + a, secs + b
    finally:
        st["model"].close()
    v = tok / secs
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "accepted tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            # the whole batch's step: the sample's time scaled by batch / sample sequences
            "ms_per_step": round(secs / args.steps * cfg["batch"] / st["n"] * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{cfg['shape']} W4A16 MTP spec-decode step (CPU oracle restatement)",
                       "batch_per_gpu": cfg["batch"], "global_batch": cfg["batch"], "ctx": cfg["ctx"],
                       "draft": f"chain {cfg['draft_len'] or 4}", "temperature": cfg["temperature"]},
            "cpu_baseline": {"kind": "port", "cores": os.cpu_count(), "sample": cpu_describe(cfg, st, args.steps),
                             "value": v, "unit": "accepted tokens/s"},
            "e2e": {"value": v, "unit": "accepted tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU arm
def run_gpu(args, world, rank, local, pg):
    import torch

    import specdec as S

    torch.cuda.set_device(local)
    cfg = dict(CONFIGS[args.config])
    shape = S.MODEL_SHAPES[cfg["shape"]]
    ctx = ctx_lengths(cfg, rank, world)
    extra = (args.warmup + 3 * args.steps + 8) * 65
    eng = S.Engine(shape, batch=cfg["batch"], draft_len=cfg["draft_len"] or 4, max_ctx=int(ctx.max()) + extra,
                   temperature=cfg["temperature"], top_p=1.0, seed=cfg["seed"] + 1000 * rank,
                   tree_branching=cfg["tree"], tree_nodes=64 if cfg["tree"] else 0, use_graph=True, device=local)
    eng.init_weights(cfg["seed"])
    eng.seed_state(ctx, cfg["seed"] * 7 + rank)
    stream = torch.cuda.ExternalStream(eng.stream(), device=f"cuda:{local}")
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    emitted0 = int(eng.read("emitted", np.int64, (1,))[0])
    clocks = ClockSampler(local)
    barrier(pg, local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    clocks.start()
    if args.nvtx:
        torch.cuda.nvtx.range_push("specdec_timed_steps")
    ev0.record(stream)
    for _ in range(args.steps):
        eng.step()
    ev1.record(stream)
    if args.nvtx:
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(pg, local)
    ms = ev0.elapsed_time(ev1)
    emitted1 = int(eng.read("emitted", np.int64, (1,))[0])
    tokens = emitted1 - emitted0
    ms_max = reduce_max(pg, ms, local)
    tokens_all = reduce_sum(pg, tokens, local)
    value = tokens_all / (ms_max / 1e3)
    kps = eng.info("kernels_per_step")

    # end to end through the host boundary: per step H2D of the control block,
    # graph launch, D2H of accepted lengths + emitted tokens, host sync
    B, R = cfg["batch"], eng.rows
    eng.set_active(np.ones(B, np.int32))
    e0 = int(eng.read("emitted", np.int64, (1,))[0])
    barrier(pg, local)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        eng.step_host()
    t1.record(stream)
    torch.cuda.synchronize()
    e_ms = reduce_max(pg, t0.elapsed_time(t1), local)
    e_tok = reduce_sum(pg, int(eng.read("emitted", np.int64, (1,))[0]) - e0, local)
    e2e = {"value": e_tok / (e_ms / 1e3), "unit": "accepted tokens/s", "h2d_bytes_per_step": 4 * B,
           "d2h_bytes_per_step": 4 * B + 4 * B * R, "ms_per_step": round(e_ms / args.steps, 4),
           "tokens_per_step": round(e_tok / args.steps / max(1, world), 2)}

    # verify forward (embedding .. lm_head) of graphed steps: global-timer
    # stamps around it in a second graph of the same step
    vms = [eng.step_verify_timed() for _ in range(args.steps + 1)][1:]
    verify_ms = float(np.mean(vms))
    # per-kernel-category split (eager steps with an event after every launch;
    # the intervals include each launch's latency, so they sum above a graphed step)
    prof = eng.profile(3)
    peaks, peak_src = load_peaks()
    ctx_now = eng.read("lens", np.int32, (B,)) - 0
    wbytes = eng.info("weight_bytes")
    vbytes, kvbytes, flops_per_row = workload_bytes_flops(shape, ctx_now, R, wbytes)
    M = B * R
    gemm_flops = flops_per_row * M
    gemm_tflops = gemm_flops / (prof["gemm_verify"] * 1e-3) / 1e12
    attn_gbs = kvbytes / (prof["attention"] * 1e-3) / 1e9
    # tensor peak: the burst figure when the SM clock sampled under load sat at
    # its maximum (the kernel ran unthrottled), the sustained one otherwise
    at_max = bool(clk.get("sm_mhz") and clk.get("sm_max_mhz") and clk["sm_mhz"] >= 0.97 * clk["sm_max_mhz"])
    tpeak, tsrc = ((peaks.get("bf16_tflops", 1590.0), "bf16 burst (SM clock at max under load)") if at_max
                   else (peaks.get("bf16_tflops_sustained", 1400.0), "bf16 sustained (SM clock below max)"))
    if prof["gemm_verify"] >= prof["attention"]:
        roof = {"kernel": "w4a16_tc_kernel (verify projections + lm_head)", "bound": "tensor",
                "achieved": round(gemm_tflops, 1), "peak": tpeak, "unit": "TFLOP/s",
                "peak_source": f"{peak_src} {tsrc}"}
    else:
        roof = {"kernel": "attn_tc_kernel (verify attention)", "bound": "hbm", "achieved": round(attn_gbs, 1),
                "peak": peaks.get("hbm_gbs", 6650.0), "unit": "GB/s", "peak_source": f"{peak_src} hbm copy"}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    roof["timing"] = "per-category device time of eager steps (event after every launch)"
    # DRAM bytes (read + write) of one launch from the committed ncu captures
    # (profiles/), with that launch's algorithmic bytes beside them
    if roof["bound"] == "tensor":
        roof.update(traffic=TRAFFIC["lm_head"][0], traffic_launch=TRAFFIC["lm_head"][1],
                    traffic_algorithmic=TRAFFIC["lm_head"][2])
    else:
        roof.update(traffic=TRAFFIC["attention"][0], traffic_launch=TRAFFIC["attention"][1],
                    traffic_algorithmic=TRAFFIC["attention"][2])
    verify = {"verify_us": round(verify_ms * 1e3, 1), "verify_us_source": "global-timer stamps around the forward inside a graphed step",
              "verify_bytes": vbytes,
              "verify_hbm_frac_of_measured": round(vbytes / (verify_ms * 1e-3) / 1e9 / peaks.get("hbm_gbs", 6650.0), 4),
              "verify_hbm_frac_of_8tbs": round(vbytes / (verify_ms * 1e-3) / 1e9 / 8000.0, 4),
              "verify_tflops": round(gemm_flops / (verify_ms * 1e-3) / 1e12, 1),
              "gemm_verify_tflops": round(gemm_tflops, 1), "attention_gbs": round(attn_gbs, 1),
              "profile_ms_per_step": {k: round(v, 4) for k, v in prof.items()}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and not cfg["tree"]:
        try:
            cpu = cpu_baseline(cfg)
        except Exception as exc:  # the CPU leg must not hide the GPU number
            cpu = {"value": None, "error": str(exc)[:200]}
    line = {"metric": METRIC, "value": round(value, 1), "unit": "accepted tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "w4a16 (fp16 act, fp32 acc)",
            "data": "synthetic (random int4 weights, seeded random fp16 KV)",
            "config": {"workload": f"{cfg['shape']} W4A16 MTP spec-decode step", "batch_per_gpu": B,
                       "global_batch": B * world, "ctx": int(cfg["ctx"]),
                       "draft": f"tree {cfg['tree']} 64 nodes" if cfg["tree"] else f"chain {cfg['draft_len']}",
                       "temperature": cfg["temperature"], "parallelism": f"request-sharded x{world}",
                       "l2": "inputs larger than L2 (weights + KV ~ {:.1f} GB per step)".format(vbytes / 1e9)},
            "mean_tokens_per_seq_step": round(tokens_all / (args.steps * B * world), 3),
            "e2e": e2e, "gpu_launches": kps * args.steps, "clocks": clk, "roofline": roof, "verify": verify,
            "cpu_baseline": cpu}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


# ------------------------------------------------------------ prefill
def run_prefill(args):
    """Chunked prefill of the engine (64-token verify forwards over the paged
    KV): `--kernel prefill --shape model,batch,prompt_len` (default
    llama3-8b,32,2048), random-init weights and uniform random prompts; prints the
    prompt tokens per second of `--steps` timed prefills (each into a fresh
    KV after `specdec_engine_retire` of every slot) after `--warmup`."""
    import torch

    import specdec as S

    parts = (args.shape or "llama3-8b,32,2048").split(",")
    model, B, P = parts[0], int(parts[1]), int(parts[2])
    shape = S.MODEL_SHAPES[model]
    eng = S.Engine(shape, batch=B, draft_len=4, max_ctx=P + 64, temperature=0.8, seed=1, use_graph=False)
    eng.init_weights(1)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, shape["vocab"], (B, P)).astype(np.int32)

    def one():
        for b in range(B):
            eng.retire(b)
        eng.prefill(prompts)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(torch.cuda.ExternalStream(eng.stream()))
    for _ in range(args.steps):
        one()
    e1.record(torch.cuda.ExternalStream(eng.stream()))
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    toks = B * (P - 1)
    print(json.dumps({"kernel": "prefill", "model": model, "batch": B, "prompt_len": P, "ms_per_prefill": round(ms, 3),
                      "prompt_tokens_per_s": round(toks / (ms / 1e3), 1), "chunk_rows": 64 * B,
                      "timing": "CUDA events on the engine stream around --steps prefills (host-synchronised calls)"}),
          flush=True)
    eng.close()


# ------------------------------------------------------------ single-kernel mode
def run_kernel(args):
    """One hot kernel on synthetic inputs, for profiler captures: `--kernel gemm
    --shape M,N,K` (W4A16 GEMM, random int4 weights), `--kernel attention
    --shape B,R,Hq,Hkv,hd,ctx` (verify attention over a shuffled paged KV pool)
    or `--kernel accept --shape B,k,V,T,top_p` (chain acceptance on fp32 logits;
    default the acceptance micro-benchmark 256,7,128256,0.7,0.9).
    Runs `--warmup` launches, then times `--steps` launches replayed from one
    CUDA graph and prints the mean time per launch; this is a kernel timing,
    not the benchmark metric."""
    import ctypes as C

    import torch

    import specdec as S

    L = S.lib()
    g = torch.Generator(device="cuda").manual_seed(0)
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    cur = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    if args.kernel == "accept":
        # chain acceptance on fp32 logits: target N(0, 3) [B, k+1, V], draft =
        # target + N(0, 0.5) [B, k, V], drafts = the draft rows' arg-max
        parts = (args.shape if args.shape.count(",") == 4 else "256,7,128256,0.7,0.9").split(",")
        B, k, V = (int(x) for x in parts[:3])
        T, tp = float(parts[3]), float(parts[4])
        ga = torch.Generator(device="cuda").manual_seed(4)
        tgt = torch.randn((B, k + 1, V), device="cuda", generator=ga) * 3
        dr = tgt[:, :k] + torch.randn((B, k, V), device="cuda", generator=ga) * 0.5
        drafts = dr.argmax(-1).to(torch.int32).contiguous()
        acc = torch.empty(B, dtype=torch.int32, device="cuda")
        out = torch.empty((B, k + 1), dtype=torch.int32, device="cuda")
        ws_b = L.specdec_accept_workspace_bytes(B * (2 * k + 1))
        ws = torch.empty(ws_b, dtype=torch.uint8, device="cuda")
        sp = S.sampling(T, tp, 4, 0)
        call = lambda: L.specdec_accept_chain(ptr(tgt), ptr(dr), ptr(drafts), B, k, V, C.byref(sp),  # noqa: E731
                                              ptr(acc), ptr(out), ptr(ws), ws_b, cur())
        algo = {"bytes": (2 * k + 1) * B * V * 4}
        args.shape = f"{B},{k},{V},{T},{tp}"
    dims = [int(x) for x in args.shape.split(",")] if args.kernel != "accept" else []
    if args.kernel in ("gemm", "gemm_tc", "gemv"):
        M, N, K = dims
        packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
        scales = (torch.rand((N, (K + 127) // 128), device="cuda", generator=g) * 0.01 + 0.001).half()
        nbytes = L.specdec_w4_tiled_bytes(N, K)
        # enough weight copies that consecutive launches read them from HBM, not L2
        copies = max(1, -(-300_000_000 // nbytes))
        tiled = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        for t in tiled:
            S.check(L.specdec_w4_tile(ptr(packed), ptr(scales), N, K, ptr(t), None))
        X = torch.randn((M, K), device="cuda", generator=g).half()
        Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        rot = {"i": 0}

        def wnext():
            rot["i"] += 1
            return ptr(tiled[rot["i"] % copies])

        if args.kernel == "gemm_tc":  # the tcgen05 tiles on the planner's plan (or --plan), whatever M
            plan = (C.c_int32 * 4)()
            S.check(L.specdec_w4a16_plan(M, N, K, 0, plan))
            qn, split = (int(plan[1]), int(plan[2])) if not args.plan else (int(x) for x in args.plan.split(","))
            args.shape += f" plan {qn},{split}"
            call = lambda: L.specdec_w4a16_gemm_with_plan(ptr(X), M, K, wnext(), N, K, ptr(Y), N, 0,  # noqa: E731
                                                          qn, split, cur())
        elif args.kernel == "gemv":
            call = lambda: L.specdec_w4a16_gemv(ptr(X), M, K, wnext(), N, K, ptr(Y), N, 0, cur())  # noqa: E731
        else:  # as the planner routes it
            call = lambda: L.specdec_w4a16_gemm(ptr(X), M, K, wnext(), N, K, ptr(Y), N, 0, None, 0, cur())  # noqa: E731
        algo = {"bytes": N * K // 2 + N * ((K + 127) // 128) * 2, "flops": 2.0 * M * N * K}
    elif args.kernel == "attention":
        B, R, Hq, Hkv, hd, ctx = dims
        max_blocks = (ctx + R + 15) // 16 + 1
        nblk = B * max_blocks
        pool = (torch.randn((nblk, 2, Hkv, 16, hd), device="cuda", generator=g) * 0.5).half()
        perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(1)).to("cuda", torch.int32)
        tables = perm.reshape(B, max_blocks).contiguous()
        ctxs = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        causal = np.array([(1 << (r + 1)) - 1 for r in range(R)], dtype=np.uint64)  # row r sees new keys 0..r
        mask = torch.from_numpy(causal.view(np.int64)).to("cuda")
        q = torch.randn((B * R, Hq, hd), device="cuda", generator=g).half()
        out = torch.empty_like(q)
        call = lambda: L.specdec_attention(ptr(q), ptr(pool), nblk, Hkv, hd, ptr(tables), max_blocks,  # noqa: E731
                                           ptr(ctxs), ptr(mask), B, R, Hq, ptr(out), None, 0, cur())
        algo = {"bytes": B * Hkv * (ctx + R) * hd * 2 * 2}
    # warm-up launches, then `steps` launches captured once in a CUDA graph and
    # replayed: the device time per launch without the host's launch path
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            S.check(call())
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.steps):
            S.check(call())
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / args.steps * 1e3
    res = {"kernel": args.kernel, "shape": args.shape, "us_per_launch": round(us, 2),
           "gbs_algorithmic": round(algo["bytes"] / us / 1e3, 1)}
    if "flops" in algo:
        res["tflops"] = round(algo["flops"] / us / 1e6, 1)
    peaks, src = load_peaks()
    res["hbm_frac"] = round(algo["bytes"] / us / 1e3 / peaks["hbm_gbs"], 3)
    res["hbm_peak_gbs"] = peaks["hbm_gbs"]
    res["peak_source"] = src
    if args.kernel == "accept":
        res["mean_accepted"] = round(float(acc.float().mean()), 3)
    print(json.dumps(res), flush=True)


def run_accept_sharded(args):
    """The acceptance micro-benchmark with the vocabulary split across the
    ranks of a torchrun job (one GPU each, NCCL): rank r holds columns
    [v0, v0 + Vs) of every logits row and the ranks exchange per-row
    statistics only (specdec.dist.accept_chain_vocab_sharded).  Times the
    whole sharded acceptance, collectives included, as the slowest rank's
    device time."""
    import torch

    import specdec as S
    from specdec.dist import TorchComm, accept_chain_vocab_sharded, vocab_shard

    world, rank, local, pg = dist_setup()
    try:
        torch.cuda.set_device(local)
        parts = (args.shape if args.shape.count(",") == 4 else "256,7,128256,0.7,0.9").split(",")
        B, k, V = (int(x) for x in parts[:3])
        T, tp = float(parts[3]), float(parts[4])
        v0, vs = vocab_shard(V, world, rank)
        g = torch.Generator(device="cuda").manual_seed(4 + 1000 * rank)
        tgt = torch.randn((B, k + 1, vs), device="cuda", generator=g) * 3
        dr = tgt[:, :k] + torch.randn((B, k, vs), device="cuda", generator=g) * 0.5
        comm = TorchComm(torch.distributed)
        # drafts = the draft rows' arg-max over the whole vocabulary (as the
        # single-GPU micro-benchmark), from the ranks' shard maxima
        L = S.lib()
        import ctypes as C

        pt = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        mx = torch.empty(B * k, dtype=torch.float32, device="cuda")
        am = torch.empty(B * k, dtype=torch.int32, device="cuda")
        drc = dr.contiguous()
        S.check(L.specdec_shard_row_max(pt(drc), B * k, None, 0, vs, v0, pt(mx), pt(am), st))
        gm, ga = comm.all_gather(mx), comm.all_gather(am)
        S.check(L.specdec_shard_merge_max(pt(gm), pt(ga), world, B * k, pt(mx), pt(am), st))
        drafts = am.view(B, k).contiguous()
        sp = S.sampling(T, tp, 4, 0)
        # the captured form (one CUDA graph of the kernels and collectives per
        # call) where it applies; its result is checked against the
        # host-issued sequence once
        captured = None
        if T > 0.0 and tp < 1.0 and world <= 8:
            from specdec.dist import ShardedChainAcceptor

            tgt, dr = tgt.contiguous(), dr.contiguous()
            captured = ShardedChainAcceptor(tgt, dr, drafts, k, v0, sp, comm, graph=True)
            a1, o1 = captured(0)
            a2, o2 = accept_chain_vocab_sharded(tgt, dr, drafts, k, v0, sp, comm)
            same = bool(torch.equal(a1, a2) and torch.equal(o1, o2))
        call = (lambda: captured(0)) if captured is not None else (
            lambda: accept_chain_vocab_sharded(tgt, dr, drafts, k, v0, sp, comm))
        try:
            for _ in range(args.warmup):
                call()
            torch.cuda.synchronize()
            barrier(pg, local)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                acc, _ = call()
            e1.record()
            torch.cuda.synchronize()
        finally:
            if captured is not None:
                captured.close()  # a graph holding collectives must go before the process group
                captured = None
                torch.cuda.synchronize()
        us = reduce_max(pg, e0.elapsed_time(e1) / args.steps * 1e3, local)
        if rank == 0:
            peaks, src = load_peaks()
            total = (2 * k + 1) * B * V * 4
            print(json.dumps({"kernel": "accept (vocabulary-sharded)", "shape": f"{B},{k},{V},{T},{tp}",
                              "n_gpus": world, "us_per_launch": round(us, 2),
                              "issue": "one CUDA graph per call" if T > 0.0 and tp < 1.0 and world <= 8
                              else "host-issued kernels and collectives",
                              "graph_matches_host_issued": same if T > 0.0 and tp < 1.0 and world <= 8 else None,
                              "gbs_algorithmic_per_gpu": round(total / world / us / 1e3, 1),
                              "hbm_frac_per_gpu": round(total / world / us / 1e3 / peaks["hbm_gbs"], 3),
                              "mean_accepted": round(float(acc.float().mean()), 3)}), flush=True)
    finally:
        if pg is not None:
            pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="8b", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--nvtx", action="store_true", help="mark the timed steps with an NVTX range (profiler filter)")
    ap.add_argument("--kernel", choices=["gemm", "gemm_tc", "gemv", "attention", "accept", "prefill"],
                    help="time one hot kernel instead of the step (gemm: as the planner routes it; gemm_tc: the "
                         "tcgen05 tiles; gemv: the few-row kernel)")
    ap.add_argument("--plan", default="", help="--kernel gemm_tc: units per CTA and k split, e.g. 2,8")
    ap.add_argument("--shape", default="160,128256,4096",
                    help="--kernel shape: M,N,K (gemm), B,R,Hq,Hkv,hd,ctx (attention) or B,k,V,T,top_p (accept)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.kernel == "accept" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_accept_sharded(args)
        return
    if args.kernel == "prefill":
        run_prefill(args)
        return
    if args.kernel:
        run_kernel(args)
        return
    if args.impl == "reference":
        # CPU arm: rank 0 alone measures; other ranks exit without work
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local, pg = dist_setup()
    try:
        run_gpu(args, world, rank, local, pg)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
