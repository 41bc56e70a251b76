#!/usr/bin/env python
"""Benchmark of the vates_b200 hot path (one JSON line on rank 0).

Default workload (the reference's MTP-verify configuration): MTP K=3 verify decode, T=4 tokens
through 48 stacked Qwen3-Next sparse-MoE blocks (H=2048, I=512, 512 experts,
top-10, MLX 4-bit g64 experts resolved through per-layer 192-slot tables into
one packed HBM pool of 16.3 GB, shared expert). A step is the whole 48-layer
stack, ``h <- h + MoE_l(rmsnorm(h))``, replayed as one CUDA graph. The pool
is far larger than L2, so no flush is needed between steps.

``--gpus N`` under torchrun runs N independent replicas (decode does not
shard); ``value`` is the tokens all ranks processed / the slowest rank's time.
``--impl reference`` times the CPU restatement of the reference path (MLX is
not installable here) on the host cores with a bounded sample per step.
"""
from __future__ import annotations

import argparse
import contextlib
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

METRIC = "MoE tokens/s and HBM GB/s (decode T≤4); prefill tok/s at 1/2/4/8 B200"
DECODE_WORKLOAD = "decode_verify_T4_48layers_fresh_inputs"
EXPERT_BYTES = 1_769_472          # blob_layout stride at H=2048, I=512, 4-bit g64
LAYER_TRAFFIC_PER_ENTRY = 1_854_185  # dram read + write per entry (profiles/decode_moe_layer_kernel.md)
ROUTER_BYTES = 512 * 2048 * 2
SHARED_GATE_BYTES = 2048 * 2


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # wait (up to 5 s) for the first sample, which is taken before the
        # load starts and is dropped from the summary
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 5.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.05)
        return self

    @staticmethod
    def keep_busy(fn, seconds: float):
        """Replay `fn` (untimed) for about `seconds` of device time, so that
        the samples around a short timed region are taken under the same load."""
        import torch
        t0 = time.time()
        while time.time() - t0 < seconds:
            for _ in range(8):
                fn()
            torch.cuda.synchronize()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        rows = rows[1:]  # the first sample precedes the load
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "reasons": reasons, "samples": len(rows)}


@contextlib.contextmanager
def stdout_to_stderr():
    """Send file descriptor 1 to stderr while NCCL creates a communicator:
    NCCL prints its version line there, and stdout carries only the bench
    line."""
    sys.stdout.flush()
    saved_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved_fd, 1)
        os.close(saved_fd)


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        with stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ CPU legs

def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_layer_seconds(layer: int, T: int = 4, seed: int = 1) -> float:
    """CPU restatement of one layer of the benchmark stack (fresh seeded
    input, the same input, weights and routes as the GPU's layer ``layer``):
    seconds for one ``FileStreamingMoeBlock.__call__``. The seeded expert
    arrays of the routed experts are generated before the clock starts."""
    from oracle import mlx_ops as M
    from oracle import moe as OM
    from oracle import synth_np as SN
    x = SN.input_tokens(1000 * seed + layer + 1, T)
    lay = SN.LazyLayer(seed, layer)
    xn = OM.rmsnorm_unit(M.bf16(x), 1e-6)
    _, _, inds, _ = OM.router(xn, lay["wr"], 10)
    lay["pool"].prefetch(sorted(set(inds.reshape(-1).tolist())))
    t0 = time.perf_counter()
    OM.moe_block_decode(x, lay, k=10, norm_eps=1e-6, residual=x)
    return time.perf_counter() - t0


def cpu_baseline_info(sample: str, value: float, kind: str = "port") -> dict:
    return {"value": value, "unit": "tokens/s", "cores": os.cpu_count(), "kind": kind,
            "cpu_model": cpu_model(), "sample": sample}


def run_reference(args, world, rank):
    """Reference arm: the CPU restatement of the reference path (MLX, which
    the reference runs on, is not available on Linux x86). One step = one
    layer of the same 48-layer stack the GPU arm runs (layer W+i for timed
    step i, each on its own fresh input), so the expert work per step is the
    GPU's own per-layer work; tokens/s = T / (48 x mean layer time)."""
    if rank != 0:
        return 0
    L, T = args.layers, 4
    for i in range(args.warmup):
        cpu_layer_seconds(i % L, T)
    times = [cpu_layer_seconds((args.warmup + i) % L, T) for i in range(args.steps)]
    per_layer = sum(times) / len(times)
    value = T / (per_layer * L)
    sample = (f"one layer per step (layers {args.warmup % L}..{(args.warmup + args.steps - 1) % L} "
              f"of the {L}-layer fresh-input stack, T={T}); tokens/s = T / ({L} x mean layer time)")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_layer * 1e3, "ms_per_48_layer_step": per_layer * L * 1e3,
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, random-init weights)",
        "config": {"workload": DECODE_WORKLOAD, "tokens": T, "layers": L,
                   "experts": 512, "top_k": 10, "pool_slots_per_layer": 192},
        "cpu_baseline": cpu_baseline_info(sample, value),
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm

PREFILL_FLOPS_32K = 2.3365e12   # routed + shared + router FLOPs of one 32768-token layer


def run_prefill_leg(steps: int = 10, warmup: int = 3, T: int = 32768):
    """Config 2: expert-major prefill of T tokens through one layer (device
    time per call of vb_moe_prefill, inputs resident in HBM)."""
    import torch
    from vates_b200.prefill import moe_prefill
    from vates_b200.synth import config2
    _, bf16_peak, peak_kind = peaks()
    blk, x = config2(T=T)
    out = torch.empty_like(x)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(max(warmup, 3)):
        moe_prefill(blk, x, out=out, status=status)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        moe_prefill(blk, x, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    flops = PREFILL_FLOPS_32K * T / 32768
    tf = flops / (ms / 1e3) / 1e12
    res = {"workload": "prefill_32k_1layer", "tokens": T, "ms_per_step": ms,
           "tok_per_s": T / (ms / 1e3), "tflops_algorithmic": tf,
           "frac_of_bf16_peak": tf / bf16_peak, "peak_tflops": bf16_peak, "peak_kind": peak_kind,
           "status": int(status.item()), "routing": "Zipf(1.1) router bias, top-10 of 512",
           "flops_per_step": flops}
    del blk, x, out
    torch.cuda.empty_cache()
    return res


def run_prefill_ep_leg(world: int, rank: int, steps: int = 10, warmup: int = 3, T: int = 32768,
                       hot_share: float = 0.02):
    """Config 2 expert-parallel over the ranks (one per GPU) through the C ABI
    (``vb_moe_prefill_ep``, NCCL point-to-point on a communicator of its own).
    The placement comes from the route histogram of an EARLIER batch (same
    Zipf-biased router, other tokens), not of the timed one: experts with at
    least ``hot_share`` of those routes are held by every rank and computed
    there for its own tokens, the others are owned by one rank each (greedy
    LPT over their route counts). Rank r starts with tokens [r*T/N,
    (r+1)*T/N). Time = max over ranks (strong scaling, T fixed). Rank 0 also
    runs its token slice through the single-device ``vb_moe_prefill`` with
    every expert resident and reports whether the outputs are bit-identical."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from vates_b200.ep import CudaEpBackend, NativeEp, NcclComm, placement
    from vates_b200.pool import QuantPool
    from vates_b200.prefill import moe_prefill
    from vates_b200.synth import E as NE, H as HH, I as II, input_tokens, make_layer, zipf_bias
    _, bf16_peak, peak_kind = peaks()
    seed = 2
    bias = torch.from_numpy(zipf_bias(seed, NE)).cuda()
    probe = make_layer(seed, 0, QuantPool.empty_blob(1, HH, II, 4, 64, "cuda"), [], "cuda",
                       router_bias=bias)
    earlier = input_tokens(seed + 100, T)  # placement batch: not the timed input
    counts = CudaEpBackend(probe, torch.zeros(NE, dtype=torch.int32)).route(earlier)[3]
    counts = counts.cpu().numpy()
    del probe, earlier
    owner, resident = placement(counts, world, rank, share=hot_share)
    n_hot = int(((counts >= hot_share * counts.sum()) if world > 1 else np.zeros(NE, bool)).sum())
    owned = [e for e in range(NE) if resident[e]]
    pool = QuantPool.empty_blob(len(owned), HH, II, 4, 64, "cuda")
    blk = make_layer(seed, 0, pool, owned, "cuda", router_bias=bias)
    per = T // world
    x_all = input_tokens(seed, T)
    x = x_all[rank * per:(rank + 1) * per].contiguous()
    if rank != 0:
        del x_all
    with stdout_to_stderr():
        comm = NcclComm()
    ep = NativeEp(blk, owner, comm, max_tokens=per)
    out = torch.empty_like(x)
    for _ in range(max(warmup, 3)):
        ep(x, out=out)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        ep(x, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    dist.barrier()
    comm.close()
    identical = None
    if rank == 0:
        # the whole batch on one device (its reduce groups come from the
        # whole batch's routes, as the EP call's do): rank 0's rows must match
        del ep, blk, pool
        torch.cuda.empty_cache()
        full = make_layer(seed, 0, QuantPool.empty_blob(NE, HH, II, 4, 64, "cuda"), range(NE),
                          "cuda", router_bias=bias)
        ref = moe_prefill(full, x_all)[:per]
        torch.cuda.synchronize()
        identical = bool(torch.equal(ref.view(torch.int16), out.view(torch.int16)))
        del full, ref, x_all
        torch.cuda.empty_cache()
    dist.barrier()
    flops = PREFILL_FLOPS_32K * T / 32768
    tf = flops / (ms / 1e3) / 1e12
    return {"workload": "prefill_32k_1layer_ep", "tokens": T, "n_gpus": world,
            "entry": "vb_moe_prefill_ep (C ABI, NCCL send/recv)",
            "ms_per_step": ms, "tok_per_s": T / (ms / 1e3), "tflops_algorithmic": tf,
            "tflops_per_gpu": tf / world, "frac_of_bf16_peak_per_gpu": tf / world / bf16_peak,
            "peak_kind": peak_kind, "experts_per_gpu": len(owned), "hot_experts_replicated": n_hot,
            "placement": f"from an earlier batch's routes: experts with >= {hot_share:.0%} of "
                         "them on every rank, the rest LPT over their counts",
            "ep_bit_identical_reference": "rank 0's rows of vb_moe_prefill over the whole "
                                          "batch on one device",
            "ep_bit_identical": identical, "scaling": "strong"}


def run_isoquant_leg(steps: int = 20, warmup: int = 3, S: int = 131072, layers: int = 12):
    """Config 3: quantized GQA decode attention over 12 IsoQuant K4/V3 caches
    of S tokens (Hq=16, Hkv=2, D=256), one query (T=1) and an MTP verify
    block (T=4, causal). Algorithmic bytes: the packed cache read once."""
    import torch
    from vates_b200.quant_kv import AsymmetricQuantizedKVCache, asym_quantized_sdpa, build_block_so4, so4_blocks
    hbm_peak, _, peak_kind = peaks()
    g = torch.Generator(device="cuda").manual_seed(3)
    rk = so4_blocks(build_block_so4(256, seed=0))
    rv = so4_blocks(build_block_so4(256, seed=1))
    caches = []
    for _ in range(layers):
        c = AsymmetricQuantizedKVCache(64, 4, 3)
        k = torch.randn((1, 2, S, 256), generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn((1, 2, S, 256), generator=g, device="cuda").to(torch.bfloat16)
        kq, vq = c.update_and_fetch(k, v, rk=rk, rv=rv)
        caches.append((kq, vq))
        del k, v
    torch.cuda.synchronize()
    res = {"workload": "isoquant_128k_12layers", "context": S, "layers": layers}
    bytes_step = layers * 2 * S * (128 + 96 + 32)
    for T in (1, 4):
        q = torch.randn((1, 16, T, 256), generator=g, device="cuda").to(torch.bfloat16)
        ws = torch.empty(1 << 26, dtype=torch.uint8, device="cuda")
        mask = "causal" if T > 1 else None

        def step():
            for kq, vq in caches:
                asym_quantized_sdpa(q, kq, vq, 256 ** -0.5, mask, 64, 4, 3, rv=rv, workspace=ws)
        for _ in range(max(warmup, 3)):
            step()
        torch.cuda.synchronize()
        # the 12-layer step replayed as one CUDA graph (device time)
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / steps * 1e3
        del graph
        gbs = bytes_step / (us / 1e6) / 1e9
        res[f"T{T}"] = {"us_per_step": us, "hbm_gbs_algorithmic": gbs,
                        "frac_of_hbm_peak": gbs / hbm_peak, "bytes_per_step": bytes_step}
    res["peak_gbs"], res["peak_kind"] = hbm_peak, peak_kind
    del caches
    torch.cuda.empty_cache()
    return res


def run_prefill_attention_leg(steps: int = 10, warmup: int = 3, lengths=(4096, 32768)):
    """Prefill attention over a fresh IsoQuant K4/V3 cache (Hq=16, Hkv=2,
    D=256, causal, inverse V rotation fused), one layer per length: the
    tcgen05 kernel behind tiled_asymmetric_attention. Algorithmic FLOPs of the
    causal product: Hq x L(L+1)/2 visible (query, key) pairs x 4 D (QK^T and
    PV). Tensor-bound: reported against the measured bf16 peak."""
    import torch
    from vates_b200.quant_kv import (AsymmetricQuantizedKVCache, build_block_so4, so4_blocks,
                                     tiled_asymmetric_attention)
    _, tf_peak, peak_kind = peaks()
    g = torch.Generator(device="cuda").manual_seed(4)
    rk = so4_blocks(build_block_so4(256, seed=0))
    rv = so4_blocks(build_block_so4(256, seed=1))
    res = {"kernel": "kv_prefill_attn_kernel", "heads": "16 q / 2 kv", "dim": 256}
    for L in lengths:
        c = AsymmetricQuantizedKVCache(64, 4, 3)
        k = torch.randn((1, 2, L, 256), generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn((1, 2, L, 256), generator=g, device="cuda").to(torch.bfloat16)
        kq, vq = c.update_and_fetch(k, v, rk=rk, rv=rv)
        q = torch.randn((1, 16, L, 256), generator=g, device="cuda").to(torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")

        def call():
            return tiled_asymmetric_attention(q, kq, vq, scale=256 ** -0.5, mask="causal",
                                              group_size=64, k_bits=4, v_bits=3, rv=rv,
                                              status=status)
        for _ in range(max(warmup, 3)):
            call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            call()
        e1.record()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        ms = e0.elapsed_time(e1) / steps
        flops = 16 * L * (L + 1) / 2 * 4 * 256
        tfs = flops / (ms / 1e3) / 1e12
        res[f"L{L}"] = {"ms": ms, "tflops": tfs, "frac_of_bf16_peak": tfs / tf_peak,
                        "flops": flops, "tokens_per_s": L / (ms / 1e3)}
        del c, k, v, kq, vq, q
    res["peak_tflops"], res["peak_kind"] = tf_peak, peak_kind
    torch.cuda.empty_cache()
    return res


def run_decode_t1_leg(st, stream, steps: int = 20, warmup: int = 3):
    """Config 0 shape (decode, T=1) over the same 48-layer stack: token 0 of
    every layer's input. Each token is routed independently, so token 0's
    experts are among the resident ones. Bytes per layer: its distinct
    experts + the shared one + router + w_sg + x/out."""
    import torch
    hbm_peak, _, peak_kind = peaks()
    L = len(st.blocks)
    xs = [st.layer_input(l)[:1].clone() for l in range(L)]
    hs = [torch.empty((1, 2048), dtype=torch.bfloat16, device="cuda") for _ in range(L + 1)]

    def chain():
        for l, blk in enumerate(st.blocks):
            blk.decode(xs[l], out=hs[l + 1], residual=xs[l], norm_eps=st.norm_eps, stream=stream)

    with torch.cuda.stream(stream):
        chain()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    for _ in range(max(warmup, 3)):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del g
    per_layer = [len(set(r)) for r in st.token_routes(0)]
    step_bytes = sum(u * EXPERT_BYTES + EXPERT_BYTES + ROUTER_BYTES + SHARED_GATE_BYTES + 2 * 2048 * 2
                     for u in per_layer)
    gbs = step_bytes / (ms / 1e3) / 1e9
    return {"workload": "decode_T1_48layers", "ms_per_step": ms, "tokens_per_s": 1 / (ms / 1e3),
            "us_per_layer": ms * 1e3 / L, "hbm_gbs_algorithmic": gbs,
            "frac_of_hbm_peak": gbs / hbm_peak, "peak_kind": peak_kind,
            "bytes_per_step": step_bytes, "steps": steps, "warmup": max(warmup, 3)}


def _qlin_bytes(out_f: int, in_f: int) -> int:
    return out_f * in_f // 2 + out_f * (in_f // 64) * 4


def full_stack_iteration_bytes(cfg, V: int, K: int, pos: int, accepted: float) -> float:
    """Algorithmic HBM bytes of one speculative iteration of the config-4
    stack: every weight read once per pass (K drafts, the verify pass over V
    rows, the MTP sync), expected distinct experts E[U] = E (1 - (1 - k/E)^n)
    of n independent tokens (the verify's V rows; one row for a draft; the
    accepted rows for the sync), GDN states read once and written per row,
    caches read up to the current position."""
    E, k, H = cfg.experts, cfg.top_k, cfg.hidden
    expert = EXPERT_BYTES
    moe = lambda n: (E * (1 - (1 - k / E) ** n) + 1) * expert + E * H * 2 + H * 2
    gdn = _qlin_bytes(cfg.gdn_proj, H) + _qlin_bytes(H, cfg.value_dim)
    att = _qlin_bytes(cfg.attn_proj, H) + _qlin_bytes(H, cfg.attn_out)
    state = cfg.v_heads * cfg.head_v * cfg.head_k * 4
    n_gdn = sum(1 for l in range(cfg.layers) if cfg.is_linear(l))
    n_att = cfg.layers - n_gdn
    head = _qlin_bytes(cfg.vocab, H)
    verify = (n_gdn * (gdn + state * (1 + V)) + n_att * (att + cfg.kv_heads * (pos + V) * 256)
              + cfg.layers * moe(V) + head)
    mtp_layer = _qlin_bytes(H, 2 * H) + att
    mtp_cache = cfg.kv_heads * (pos + V) * 512 * 2
    draft = mtp_layer + moe(1) + head + mtp_cache
    sync = mtp_layer + moe(accepted) + mtp_cache
    return K * draft + verify + sync


def run_full_stack_leg(new_tokens: int = 128, prompt_len: int = 4096, seed: int = 4,
                       V: int = 4, K: int = 3, replays: int = 20):
    """Config 4: random-init Qwen3-Next-80B-A3B-shaped stack (48 layers: 36
    Gated-DeltaNet + 12 IsoQuant full attention, 512-expert 4-bit MoE blocks,
    vocab 151,936, MTP head), all weights resident, batch 1. A seeded
    4096-token random prompt is prefilled (chunks of V rows through the
    verify graph), then greedy MTP self-speculative decoding with K = 3
    drafts and verify at T = 4 runs for ``new_tokens`` tokens. decode_tok_s
    = generated tokens / wall time of the decode loop (host clock, one
    emitted-token counter read per iteration, as the reference's
    mtp_generate wall). Device time per iteration from CUDA events over
    back-to-back graph replays."""
    import numpy as np
    import torch
    from vates_b200.qwen_next import QwenNextConfig, QwenNextModel, SP_HIST, SP_NOUT
    hbm_peak, _, peak_kind = peaks()
    cfg = QwenNextConfig()
    cache = (prompt_len + new_tokens + 4 * replays + 256 + 255) // 256 * 256
    t0 = time.perf_counter()
    model = QwenNextModel(cfg, seed=seed, cache_len=cache, verify_len=V, drafts=K)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    rng = np.random.Generator(np.random.PCG64([seed, 4096]))
    prompt = rng.integers(0, cfg.vocab, prompt_len).astype(np.int32)
    # warm-up (captures the prefill and iteration graphs), then the measured run
    model.generate(prompt[:64], 8)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    model.prefill(prompt)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    st0 = model.buf["state"].cpu().numpy().copy()
    t0 = time.perf_counter()
    n_out = 1
    iters = 0
    g = model._graph(("iter",), lambda s: model.spec_iteration(s))
    while n_out < new_tokens:
        g.replay()
        iters += 1
        n_out = int(model.buf["state"][SP_NOUT].item())
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    st = model.buf["state"].cpu().numpy()
    toks = model.buf["out"][:new_tokens].cpu().numpy()
    hist = [int(v) for v in (st[SP_HIST:SP_HIST + V + 1] - st0[SP_HIST:SP_HIST + V + 1])]
    steps = max(sum(hist), 1)
    accepted = sum((min(m + 1, V)) * c for m, c in enumerate(hist)) / steps
    # device time: back-to-back replays without host reads
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    dev_ms = e0.elapsed_time(e1) / replays
    pos = int(st[0])
    it_bytes = full_stack_iteration_bytes(cfg, V, K, pos, accepted)
    gbs = it_bytes / (dev_ms / 1e3) / 1e9
    out = {"workload": "config4_qwen3next_48L_mtp_k3_verify_t4", "prompt_tokens": prompt_len,
           "new_tokens": int(n_out), "decode_tok_s": (n_out - 1) / wall if n_out > 1 else 0.0,
           "wall_s": wall, "iterations": iters, "tokens_per_iteration": (n_out - 1) / max(iters, 1),
           "accept_hist": hist, "ms_per_iteration_device": dev_ms,
           "bytes_per_iteration_est": it_bytes, "hbm_gbs_est": gbs,
           "frac_of_hbm_peak": gbs / hbm_peak, "peak_gbs": hbm_peak, "peak_kind": peak_kind,
           "prefill_s": prefill_s, "prefill_tok_s": prompt_len / prefill_s, "build_s": build_s,
           "status": int(model.buf["status"].item()),
           "first_tokens": [int(t) for t in toks[:8]],
           "hbm_allocated_gb": torch.cuda.memory_allocated() / 1e9,
           "note": "random-init weights: the MTP drafts rarely match, so about one token per "
                   "iteration (the reference's acceptance on trained weights is not reproducible "
                   "here)"}
    del model, g
    torch.cuda.empty_cache()
    return out


def run_residency_leg(layers: int = 8, steps: int = 12, warmup: int = 4, T: int = 4,
                      cap: int = 192, seed: int = 1):
    """Config-1 layers over a pool of ``cap`` < 512 slots per layer, misses
    loaded on demand: every step decodes a fresh seeded T-token input (new
    routes), so the miss path runs as it would for unseen tokens. All 512
    experts of each layer sit in an HBM blob store; each layer call is one
    vb_moe_decode_resident: "route_first" = a routing-only launch, read-back,
    native demand, one vb_blob_gather of the placed experts, table copy, the
    block launch; "optimistic" = the block first and again only after a miss.
    Device-timed with events over whole steps (host work between launches
    included). The gather kernel is also timed on its own: bytes = 2 x
    experts x 1,769,472 (read + write)."""
    import torch
    from vates_b200.moe_block import MoeBlock, Workspace
    from vates_b200.pool import QuantPool
    from vates_b200.residency import DeviceBlobStore, ResidentExpertPool
    from vates_b200.synth import E, H, input_tokens, make_layer
    hbm_peak, _, peak_kind = peaks()
    store_pool = QuantPool.empty_blob(layers * E, H, 512, 4, 64)
    ws = Workspace()
    src = [make_layer(seed, l, store_pool.view(l * E, E), range(E), workspace=ws)
           for l in range(layers)]
    store = DeviceBlobStore(store_pool.blob.view(layers, E, -1))
    hs = [torch.empty((T, H), dtype=torch.bfloat16, device="cuda") for _ in range(layers + 1)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    norm_eps = 1e-6
    modes = {}
    for route_first in (True, False):
        rp = ResidentExpertPool(cap, None, layers=layers, num_experts=E, hidden=H, inter=512,
                                blob_store=store)
        blocks = [MoeBlock(b.router_w, rp.tables[l], rp.layer_pool(l), b.shared,
                           b.shared_gate_w, top_k=b.top_k, workspace=ws)
                  for l, b in enumerate(src)]
        dbg = blocks[0].new_debug(T)
        runs = [0]

        def step(i):
            hs[0].copy_(input_tokens(seed * 1000 + i, T))
            for l in range(layers):
                runs[0] += rp.decode(l, blocks[l], hs[l], hs[l + 1], residual=hs[l],
                                     status=status, debug=dbg, norm_eps=norm_eps,
                                     route_first=route_first)

        for i in range(warmup):
            step(i)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        h0, m0 = rp.hits, rp.misses
        runs[0] = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            step(warmup + i)
        e1.record()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        ms = e0.elapsed_time(e1) / steps
        hits, misses = rp.hits - h0, rp.misses - m0
        modes["route_first" if route_first else "optimistic"] = {
            "ms_per_step": ms, "tokens_per_s": T / (ms / 1e3), "us_per_layer": ms * 1e3 / layers,
            "unique_expert_hits": hits, "unique_expert_misses": misses,
            "miss_rate": misses / max(hits + misses, 1),
            "experts_loaded_per_step": misses / steps,
            "kernel_launches_per_layer": runs[0] / (steps * layers)}
        keep = rp
        del blocks

    # The gather kernel alone: 24 experts (about one T=4 layer's misses) into
    # slots of layer 0, device-resident indices, CUDA events around each launch;
    # 85 MB per launch from a different source layer each time (inputs > L2).
    from vates_b200._lib import check, lib
    n_g, reps = 24, 20
    lp = keep.layer_pool(0)
    idx = [torch.tensor([[(r * 37 + j * 11) % E for j in range(n_g)],
                         [lp.blob_slot0 + (r * 5 + j) % cap for j in range(n_g)]],
                        dtype=torch.int32, device="cuda") for r in range(reps)]

    def gather(r):
        check(lib.vb_blob_gather(store.blobs[r % layers].data_ptr(), store.stride,
                                 idx[r][0].data_ptr(), idx[r][1].data_ptr(), n_g,
                                 lp.blob.data_ptr(), torch.cuda.current_stream().cuda_stream),
              "vb_blob_gather")

    for r in range(3):
        gather(r)
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gather_ms = 0.0
    for r in range(reps):
        g0.record()
        gather(r)
        g1.record()
        g1.synchronize()
        gather_ms += g0.elapsed_time(g1)
    gather_ms /= reps
    gbytes = 2 * n_g * EXPERT_BYTES
    gbs = gbytes / (gather_ms / 1e3) / 1e9
    del keep, store, store_pool, src
    torch.cuda.empty_cache()
    return {"workload": f"decode_T{T}_{layers}layers_pool{cap}_of_{E}_fresh_tokens",
            "modes": modes,
            "blob_gather": {"kernel": "blob_gather_kernel", "experts": n_g, "bytes": gbytes,
                            "ms": gather_ms, "gbs": gbs, "frac_of_hbm_peak": gbs / hbm_peak,
                            "peak_kind": peak_kind},
            "steps": steps, "warmup": warmup}


def decode_stack_graph(st, stream):
    """The whole 48-layer step of ``st`` captured as one CUDA graph."""
    import torch
    with torch.cuda.stream(stream):  # warm the kernels (attribute setup) outside capture
        st.step(stream=stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        st.step(stream=stream)
    torch.cuda.synchronize()
    return graph


def time_graph(graph, steps: int, warmup: int) -> float:
    import torch
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def step_bytes_of(U, T: int) -> int:
    """Algorithmic HBM bytes of one stack step: per layer the distinct routed
    experts and the shared one (1,769,472 B each), the router (2 MiB), the
    shared-expert gate, and x, residual and out (T x H bf16 each)."""
    return sum(u * EXPERT_BYTES + EXPERT_BYTES + ROUTER_BYTES + SHARED_GATE_BYTES
               + 3 * T * 2048 * 2 for u in U)


def run_decode_chain_leg(stream, steps: int = 20, warmup: int = 3, T: int = 4, L: int = 48):
    """The same stack as a chain (layer l+1's input is layer l's output): with
    random-init weights the chain routes fewer distinct experts per layer, so
    a step reads fewer bytes."""
    import torch
    from vates_b200.synth import DecodeStack
    hbm_peak, _, peak_kind = peaks()
    st = DecodeStack(seed=1, layers=L, cap=192, T=T, fresh=False)
    st.ensure_resident()
    U = st.unique_experts()
    graph = decode_stack_graph(st, stream)
    ms = time_graph(graph, steps, warmup)
    del graph
    sb = step_bytes_of(U, T)
    gbs = sb / (ms / 1e3) / 1e9
    del st
    torch.cuda.empty_cache()
    return {"workload": f"decode_verify_T{T}_{L}layers_chain", "ms_per_step": ms,
            "tokens_per_s": T / (ms / 1e3), "unique_experts_per_layer": U,
            "unique_experts_per_layer_mean": sum(U) / len(U), "bytes_per_step": sb,
            "hbm_gbs_algorithmic": gbs, "frac_of_hbm_peak": gbs / hbm_peak,
            "peak_kind": peak_kind}


def run_decode(args, world, rank, local):
    import torch
    from vates_b200.synth import DecodeStack

    hbm_peak, _, peak_kind = peaks()
    T, L = 4, args.layers
    st = DecodeStack(seed=1, layers=L, cap=192, T=T, fresh=True)
    st.ensure_resident()
    U = st.unique_experts()
    torch.cuda.synchronize()

    stream = torch.cuda.Stream()
    graph = decode_stack_graph(st, stream)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    # ---- timed region: K graph replays (device time, max over ranks) ----
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The sampler runs from 0.5 s of untimed replays before the timed region
    # to 0.5 s after it: nvidia-smi samples every 100 ms, and the timed
    # region alone is shorter than that.
    with ClockSampler(local) as clk:
        ClockSampler.keep_busy(graph.replay, 0.5)
        barrier(world)
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
        barrier(world)
        ClockSampler.keep_busy(graph.replay, 0.5)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms, world)
    clocks = clk.summary()
    value = world * T / (ms / 1e3)

    # ---- end to end through the public API with host buffers: every step
    # copies its 48 layer inputs from pinned host memory and reads the last
    # layer's output back ----
    x_host = torch.empty(tuple(st.xs.shape), dtype=torch.bfloat16, pin_memory=True)
    x_host.copy_(st.xs.cpu())
    y_host = torch.empty((T, 2048), dtype=torch.bfloat16, pin_memory=True)
    cur = torch.cuda.current_stream()
    for _ in range(3):
        st.xs.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(st.hs[-1], non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        st.xs.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(st.hs[-1], non_blocking=True)
    e1.record(cur)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    barrier(world)

    # ---- warm in-graph kernel spans from the kernel's %globaltimer trace ----
    trace = torch.empty((L, 16), dtype=torch.int64, device="cuda")
    init = torch.tensor([-1, 0] + [0] * 14, dtype=torch.int64, device="cuda")
    tgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(tgraph, stream=stream):
        st.step(stream=stream, trace=trace)
    for _ in range(3):
        trace.copy_(init.expand(L, 16))
        tgraph.replay()
        torch.cuda.synchronize()
    tr = trace.cpu().numpy().astype("uint64").astype("float64")
    del tgraph
    kspan = (tr[:, 1] - tr[:, 0]).mean() / 1e3
    layer_us = (tr[1:, 0] - tr[:-1, 0]).mean() / 1e3
    marks = {name: (tr[:, m] - tr[:, 0]).mean() / 1e3 for m, name in (
        (2, "pdl_wait"), (3, "router_rows"), (4, "grid_barrier"), (9, "route_max"),
        (10, "route_sum"), (11, "route_candidates"), (12, "route_topk"), (5, "routing"),
        (6, "gateup"), (7, "down"), (8, "combine"))}

    # ---- the layer kernel timed per launch with CUDA events outside the
    # graph and the PDL chain (each launch starts cold) ----
    evs, arr = st.blocks[0].timing_events()
    cold_ms = 0.0
    reps = 3
    for _ in range(reps):
        for l, blk in enumerate(st.blocks):
            xin = st.layer_input(l)
            blk.decode(xin, out=st.hs[l + 1], residual=xin, norm_eps=st.norm_eps, timing=arr)
            evs[1].synchronize()
            cold_ms += evs[0].elapsed_time(evs[1])
    cold_ms /= reps * L

    step_bytes = step_bytes_of(U, T)
    hbm_gbs = step_bytes / (ms / 1e3) / 1e9
    layer_bytes = step_bytes / L  # per launch, algorithmic
    # The timed region holds nothing but the 48 launches of the layer kernel
    # per step, so its average launch takes ms / L.
    launch_ms = ms / L
    achieved = layer_bytes / (launch_ms / 1e3) / 1e9
    # DRAM traffic per launch: an ncu capture of the 4-layer fresh-input case
    # read+wrote LAYER_TRAFFIC_PER_ENTRY bytes per entry (routed experts + the
    # shared one); scaled to this run's mean entries per launch.
    traffic = LAYER_TRAFFIC_PER_ENTRY * (sum(U) / L + 1)

    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, random-init weights)",
        "config": {"workload": DECODE_WORKLOAD, "tokens": T, "layers": L,
                   "hidden": 2048, "inter": 512, "experts": 512, "top_k": 10,
                   "pool_slots_per_layer": 192, "quant": "mlx affine 4-bit g64",
                   "inputs": "a fresh seeded N(0,1) input per layer (independent routes)",
                   "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2 (16.3 GB pool, ~3.5 GB read per step)"},
        "hbm_gbs_algorithmic": hbm_gbs,
        "hbm_frac_of_measured": hbm_gbs / hbm_peak,
        "hbm_frac_of_8tbs": hbm_gbs / 8000.0,
        "bytes_per_step": step_bytes,
        "unique_experts_per_layer": U,
        "unique_experts_per_layer_mean": sum(U) / len(U),
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(st.xs.numel() * 2), "d2h_bytes_per_step": T * 2048 * 2},
        "roofline": {"kernel": "moe_layer_kernel", "bound": "hbm", "achieved": achieved,
                     "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "traffic_unit": "bytes per launch",
                     "bytes_per_launch": layer_bytes, "ms_per_launch": launch_ms,
                     "cold_launch_ms": cold_ms,
                     "cold_launch_gbs": layer_bytes / (cold_ms / 1e3) / 1e9},
        "kernel_trace_us": {"span": kspan, "layer_period": layer_us,
                            "marks_from_start": marks},
        "gpu_launches": L * args.steps,
        "clocks": clocks,
    }
    del graph
    if not args.no_extra:
        out["decode_t1"] = run_decode_t1_leg(st, stream)
        del st
        torch.cuda.empty_cache()
        out["decode_chain"] = run_decode_chain_leg(stream)
        if world == 1:
            out["prefill"] = run_prefill_leg()
            out["isoquant"] = run_isoquant_leg()
            out["prefill_attention"] = run_prefill_attention_leg()
            out["residency"] = run_residency_leg()
            out["full_stack"] = run_full_stack_leg()
        else:
            out["prefill"] = run_prefill_ep_leg(world, rank)
    if rank == 0 and world == 1 and not args.no_cpu:
        secs = [cpu_layer_seconds(l, T) for l in range(args.cpu_layers)]
        cpu_tok_s = T / (sum(secs) / len(secs) * L)
        out["cpu_baseline"] = cpu_baseline_info(
            f"layers 0..{args.cpu_layers - 1} of the {L}-layer fresh-input stack (the GPU's own "
            f"inputs and routes), T={T}; tokens/s = T / ({L} x mean layer time)", cpu_tok_s)
    if rank == 0:
        print(json.dumps(out), flush=True)
    return 0


def _fresh_stack(layers: int):
    """The headline decode stack (fresh seeded inputs per layer, T = 4)."""
    from vates_b200.synth import DecodeStack
    st = DecodeStack(seed=1, layers=layers, cap=192, T=4, fresh=True)
    st.ensure_resident()
    return st


def torch_stream():
    import torch
    return torch.cuda.Stream()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode"])
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--cpu-layers", type=int, default=4)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the prefill (config 2) and IsoQuant (config 3) legs")
    ap.add_argument("--leg", default=None,
                    choices=["prefill", "isoquant", "prefill_attention", "residency",
                             "full_stack", "decode_t1"],
                    help="run only this extra leg on one GPU and print its result (for profiling)")
    ap.add_argument("--iso-layers", type=int, default=12)
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.leg is not None:
        legs = {"prefill": lambda: run_prefill_leg(args.steps, args.warmup),
                "isoquant": lambda: run_isoquant_leg(args.steps, args.warmup,
                                                     layers=args.iso_layers),
                "prefill_attention": lambda: run_prefill_attention_leg(args.steps, args.warmup),
                "residency": lambda: run_residency_leg(),
                "full_stack": lambda: run_full_stack_leg(),
                "decode_t1": lambda: run_decode_t1_leg(
                    _fresh_stack(args.layers), torch_stream(), args.steps, args.warmup)}
        print(json.dumps({args.leg: legs[args.leg]()}), flush=True)
        return 0
    try:
        if args.impl == "reference":
            rc = run_reference(args, world, rank)
        else:
            rc = run_decode(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
