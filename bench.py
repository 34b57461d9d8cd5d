"""Benchmark: E8 + rANS KV-cache encode -> full decode.

Workload (per rank, weak scaling): a Llama-3.1-8B-shaped KV cache, 32 layers
x 8 KV heads x head_dim 128, batch 1, seq 8192, bf16; K = N(0,1) * exp(N(0,1))
per (layer, head, channel) with one outlier channel x10 per (layer, head)
(1% of 128), V = N(0,1); 4 bits/dim.  One chunk per (layer, K/V) as the
reference's prefill makes them (llm/compressed_kv_cache.py:360-361): 64 chunks
of 8 heads x 131072 E8 blocks = 67,108,864 blocks per step.

A step = encode every chunk (scales, E8 + symbols, tables, rANS lanes) and
decode every chunk back to bf16.  value = E8 blocks round-tripped per second
(Gvec/s), inputs resident in HBM (1 GiB > L2, so no flush is needed).
e2e = the same through the public API from pinned host memory: H2D of the
bf16 cache, compress, decompress, D2H of the decoded cache.

The line also carries "attention": BASELINE config 3, one fused dequant +
decode-attention step (B=16, 32 query / 8 KV heads, head_dim 128, context
32768 compressed at 4 bits/dim; K/V = N(0,1) * lognormal(0, 0.5) per vector,
q ~ N(0, 1/sqrt(128)) bf16), metric = algorithmic bytes (compressed K+V +
lane metadata + q + o) per second.  At N GPUs the context is sequence-sharded:
each rank attends over its slice and one NCCL all-gather of (o, lse) plus the
LSE merge completes the step (strong scaling of one decode step).

"config4" carries BASELINE config 4: a Qwen2.5-7B-shaped mixed-rate cache
(28 layers x 4 KV heads x head_dim 128, batch 4, context 131072; per-layer
bits from {3, 4, 5} with exactly 3 layers at 5; K ~ Student-t(3), V ~ N(0,1)),
whole-model encode and one fused decode-attention step over every layer,
sharded by (layer, KV head) units over the ranks with no collective.  The
line reports how many tokens went to the outlier side channel (chunks whose
alphabet would exceed L = 1024 symbols).

"config1" carries BASELINE config 1: 262,144 vectors of dim 128, fp32
N(0,1) with a log-normal(0, 0.5) magnitude per vector, one fp16 scale per
vector (the reference's _compress_tensor of the (1, 262144, 1, 128) view,
llm/compressed_kv_cache.py:176-196), 4 bits/dim: encode + decode Gvec/s,
reconstructed MSE and bitstream bytes, beside the C oracle's values for the
same seeded input (rank 0 at N = 1).

"config5" carries BASELINE config 5: a random-init Llama-3.1-8B-architecture
model decoding through CompressedAttentionKVCache (batch 32, prefill 16,384
random ids, 256 generated tokens, 4 bits/dim, KV-head-sharded at N > 1):
decode tokens/s, the fused attention's share of a step and its roofline.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_LAYERS, N_KV, SEQ, HD, BITS = 32, 8, 8192, 128, 4
N_CHUNKS = 2 * N_LAYERS
BPH = SEQ * HD // 8
BLOCKS = N_CHUNKS * N_KV * BPH
TILE = 1024
E2E_GROUP = 1  # chunks per pipelined e2e transfer group
METRIC = "E8+rANS encode/decode Gvec/s"
UNIT = "Gvec/s"
# config 3 (fused dequant + decode attention)
A_B, A_HKV, A_G, A_S, A_D = 16, 8, 4, 32768, 128
A_METRIC = "fused dequant-attn HBM GB/s"
# config 4 (Qwen2.5-7B-shaped mixed-rate cache)
C4_LAYERS, C4_KV, C4_B, C4_S, C4_D, C4_G = 28, 4, 4, 131072, 128, 7
# DRAM bytes (read + write) per E8 block of each codec phase and per
# compressed byte of the attention kernel, measured with ncu
# (dram__bytes_read.sum + dram__bytes_write.sum) on the 8-layer config-2 case
# (decode: the full-size capture, whose bf16 output no longer fits L2) and
# the full config-3 step (rANS lanes; compact layout: 943.4 MB read + 13.8 MB
# written against 937.0 MB algorithmic); scaled to each launch for
# roofline.traffic.
TRAFFIC_PER_BLOCK = {"scales": 16.0, "quantize": 23.0, "encode": 20.6, "decode": 20.2}
ATTN_TRAFFIC_PER_ALG_BYTE = 602.4 / 583.6
COMPACT_TRAFFIC_PER_ALG_BYTE = (943.4 + 13.8) / 937.0


def make_cache(gen_device, seed, n_layers=N_LAYERS):
    """Synthetic config-2 K/V, chunk c = 2*layer + (0: K, 1: V) -> (2*layers, 8, 8192, 128) bf16."""
    import torch

    g = torch.Generator(device=gen_device)
    g.manual_seed(1000 + seed)
    x = torch.empty(2 * n_layers, N_KV, SEQ, HD, dtype=torch.bfloat16, device=gen_device)
    for layer in range(n_layers):
        s_c = torch.exp(torch.randn(N_KV, 1, HD, generator=g, device=gen_device))
        out_ch = torch.randint(0, HD, (N_KV,), generator=g, device=gen_device)
        s_c[torch.arange(N_KV, device=gen_device), 0, out_ch] *= 10.0
        x[2 * layer] = (torch.randn(N_KV, SEQ, HD, generator=g, device=gen_device) * s_c).to(torch.bfloat16)
        x[2 * layer + 1] = torch.randn(N_KV, SEQ, HD, generator=g, device=gen_device).to(torch.bfloat16)
    return x


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [p.strip() for p in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_baseline(n_threads, sample_chunks=2, reps=1, min_seconds=0.0):
    """The C oracle port (oracle/lq_oracle_codec.c) on a bounded sample of the
    workload: `sample_chunks` config-2 chunks coded and decoded `reps` times,
    or more often until `min_seconds` have passed."""
    import numpy as np

    import oracle.lq_oracle as O

    O.build()
    rng = np.random.default_rng(7)
    x = np.empty((sample_chunks, N_KV, SEQ, HD), np.float32)
    for c in range(sample_chunks):
        if c % 2 == 0:
            s_c = np.exp(rng.standard_normal((N_KV, 1, HD))).astype(np.float32)
            s_c[np.arange(N_KV), 0, rng.integers(0, HD, N_KV)] *= 10.0
            x[c] = rng.standard_normal((N_KV, SEQ, HD)).astype(np.float32) * s_c
        else:
            x[c] = rng.standard_normal((N_KV, SEQ, HD)).astype(np.float32)
    # bf16 bit patterns (round to nearest even)
    u = x.view(np.uint32)
    xb = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    t0 = time.perf_counter()
    done = 0
    while done < reps or (time.perf_counter() - t0 < min_seconds and done < 64):
        O.codec_roundtrip_batch(xb, O.DT_BF16, sample_chunks, N_KV, BPH, BITS, TILE, O.DT_BF16, n_threads)
        done += 1
    dt = time.perf_counter() - t0
    blocks = done * sample_chunks * N_KV * BPH
    return blocks / dt / 1e9, blocks, dt


def attention_kv(gen_device, seed, s_len):
    """Config-3 K or V slice: N(0,1) * lognormal(0, 0.5) per vector, bf16."""
    import torch

    g = torch.Generator(device=gen_device)
    g.manual_seed(seed)
    shape = (A_B, A_HKV, s_len, A_D)
    return (torch.randn(shape, generator=g, device=gen_device) *
            torch.exp(0.5 * torch.randn(A_B, A_HKV, s_len, 1, generator=g, device=gen_device))).to(torch.bfloat16)


def attention_query(gen_device):
    import torch

    g = torch.Generator(device=gen_device)
    g.manual_seed(3003)
    return (torch.randn(A_B, A_HKV * A_G, A_D, generator=g, device=gen_device) / A_D ** 0.5).to(torch.bfloat16)


def cpu_attention_baseline(s_len=2048):
    """Reference CPU path of one decode step on a sample: oracle lane decode +
    dequant (oracle/lq_oracle_codec.c) of K and V for one batch row, then the
    softmax attention in numpy; rate in GB/s of the same algorithmic bytes."""
    import numpy as np

    import oracle.lq_oracle as O

    O.build()
    rng = np.random.default_rng(11)
    shape = (1, A_HKV, s_len, A_D)
    chunks = []
    for _ in range(2):
        x = (rng.standard_normal(shape) * np.exp(0.5 * rng.standard_normal(shape[:3] + (1,)))).astype(np.float32)
        chunks.append(O.compress_chunk(x, O.DT_F32, A_HKV, s_len * A_D // 8, BITS, TILE))
    q = (rng.standard_normal((1, A_HKV * A_G, A_D)) / A_D ** 0.5).astype(np.float32)
    t0 = time.perf_counter()
    k = O.decompress_chunk(chunks[0]).reshape(shape)
    v = O.decompress_chunk(chunks[1]).reshape(shape)
    O.decode_attention_f64(q, k, v, 1 / A_D ** 0.5)
    dt = time.perf_counter() - t0
    nbytes = sum(4 * len(c.words) + (c.n_vectors + 7) // 8 + 2 * c.n_heads for c in chunks) + 2 * q.nbytes
    return nbytes / dt / 1e9, nbytes, dt


def bench_attention(dev, rank, world, steps, warmup, barrier):
    """Config 3 on `world` ranks (sequence-sharded).  Returns the line's
    "attention" object on rank 0 (None elsewhere)."""
    import torch
    import torch.distributed as dist

    from latticequant_b200 import attention as A
    from latticequant_b200 import codec as C
    from latticequant_b200 import sharding as SH

    lo, hi = SH.sequence_slice(A_S, world, rank, TILE // (A_D // 8))
    k = attention_kv(dev, 4000 + 2 * rank, hi - lo)
    v = attention_kv(dev, 4001 + 2 * rank, hi - lo)
    q = attention_query(dev)
    kc, _ = C.compress(k, BITS, tile_blocks=TILE)
    vc, _ = C.compress(v, BITS, tile_blocks=TILE)
    del k, v
    op = A.DecodeAttention(kc, vc, A_G)
    rows = A_B * A_HKV * A_G
    # at N > 1 the kernel writes (o, lse) straight into one packed fp32 buffer,
    # all-gathered in one collective and merged from the packed layout
    packed = torch.empty(rows * A_D + rows, dtype=torch.float32, device=dev)
    o_loc = packed[:rows * A_D].view(rows, A_D) if world > 1 else \
        torch.empty(rows, A_D, dtype=torch.bfloat16, device=dev)
    l_loc = packed[rows * A_D:]
    out = torch.empty(rows, A_D, dtype=torch.bfloat16, device=dev)
    l_out = torch.empty(rows, dtype=torch.float32, device=dev)
    gathered = torch.empty(world, rows * A_D + rows, dtype=torch.float32, device=dev)

    def step():
        op(q, o_loc, l_loc if world > 1 else None)
        if world > 1:
            dist.all_gather_into_tensor(gathered, packed)
            A.merge_attention_packed(gathered, rows, A_D, out=out, lse=l_out)

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    if op.flags():
        raise RuntimeError(f"attention device error flags {op.flags():#x}")
    st = torch.cuda.current_stream(dev)
    # the fused kernel pair alone (roofline), then the whole step
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        op(q, o_loc, l_loc if world > 1 else None)
    e1.record(st)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / steps
    barrier()
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / steps
    local_bytes = (kc.compressed_bytes() + vc.compressed_bytes() + kc.metadata_bytes() + vc.metadata_bytes() +
                   q.numel() * 2 + rows * A_D * o_loc.element_size())
    comp_bytes = kc.compressed_bytes() + vc.compressed_bytes()

    # e2e: the public API call per step with host buffers (q in, o out)
    host_q = q.cpu().pin_memory()
    host_o = torch.empty(rows, A_D, dtype=torch.bfloat16).pin_memory()
    dq = torch.empty_like(q)

    def e2e_step():
        dq.copy_(host_q, non_blocking=True)
        if world > 1:
            ol, ll = A.decode_attention(dq, kc, vc, out_dtype=torch.float32, return_lse=True)
            o, _ = SH.sequence_sharded_merge(ol.view(rows, A_D), ll.view(rows), out_dtype=torch.bfloat16)
        else:
            o = A.decode_attention(dq, kc, vc)
        host_o.copy_(o.view(rows, A_D), non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0.record(st)
    k2 = max(2, min(steps, 5))
    for _ in range(k2):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1) / k2

    vals = torch.tensor([ms, k_ms, ems, float(local_bytes), float(comp_bytes)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = vals[:3].clone()
        sm = vals[3:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, sm])
    ms, k_ms, ems, tot_bytes, tot_comp = [float(t) for t in vals.tolist()]
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    achieved = local_bytes / (k_ms * 1e-3) / 1e9  # rank 0's kernel pair
    cpu = None
    try:
        v_cpu, nb, dt = cpu_attention_baseline()
        cpu = {"value": v_cpu, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"1 of {A_B} batch rows, 2048 tokens: oracle lane decode + dequant of K and V, "
                         f"numpy attention ({nb} B, {dt:.2f} s)"}
    except Exception as e:  # the baseline is reported, not required
        cpu = {"unavailable": str(e)[:200]}
    return {"metric": A_METRIC, "value": tot_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "compressed_GBps": tot_comp / (ms * 1e-3) / 1e9,
            "decode_steps_per_s": 1e3 / ms, "tokens_per_s": A_B * 1e3 / ms,
            "config": {"workload": "config3: B16 x 32 q-heads / 8 kv-heads x D128, ctx 32768, 4 b/dim, one decode "
                                   "step", "parallelism": f"sequence-sharded over {world} (one all-gather of the "
                                                          "packed (o, lse) + LSE merge)"
                                   if world > 1 else "single GPU", "tile_blocks": TILE,
                       "bits_per_dim": tot_comp * 8 / (2 * A_B * A_HKV * A_S * A_D),
                       "l2": "compressed K+V larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "attn_partial_kernel + attn_redo_kernel + attn_combine_kernel",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": local_bytes * ATTN_TRAFFIC_PER_ALG_BYTE / 1e9, "traffic_unit": "GB per launch",
                         "algorithmic_GB": local_bytes / 1e9, "kernel_ms": k_ms},
            "e2e": {"value": tot_bytes / (ems * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ems,
                    "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": rows * A_D * 2},
            "gpu_launches": steps * (3 + (1 if world > 1 else 0)), "cpu_baseline": cpu}


def c4_bits():
    """Per-layer (K, V) bits: seeded draw from {3, 4, 5} with exactly 3 layers at 5."""
    import numpy as np

    rng = np.random.default_rng(44)
    five = set(rng.choice(C4_LAYERS, 3, replace=False).tolist())
    return [5 if l in five else int(rng.choice([3, 4])) for l in range(C4_LAYERS)]


def c4_tensor(dev, seed, heads, student):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    shape = (C4_B, heads, C4_S, C4_D)
    z = torch.randn(shape, generator=g, device=dev)
    if student:  # t(3) = z / sqrt(chi2(3) / 3)
        chi = sum(torch.randn(shape, generator=g, device=dev) ** 2 for _ in range(3))
        z = z / torch.sqrt(chi / 3)
    return z.to(torch.bfloat16)


def compact_chunk_bytes(chunk):
    """Bytes the compact-layout attention kernel must read for one chunk:
    codes, fp16 fallback rows, mask words, word ranks and head scales."""
    from latticequant_b200 import attention as A

    words, rank_t = A.compact_index(chunk)
    return (chunk.packed.numel() + 2 * chunk.fallback.numel() + 4 * (words.numel() + rank_t.numel()) +
            4 * chunk.scales.numel())


def bench_attention_compact(dev, rank, world, steps, warmup, barrier):
    """Config 3 with K/V in the compact fixed-rate layout at 4 bits (the
    reference's llm/fused_triton_merge.py format: 4-byte codes + fp16
    fallback rows) and lq_attn_decode_compact, sequence-sharded at N > 1 like
    the rANS step.  Kernel-only timing through the C ABI with preallocated
    buffers; algorithmic bytes = codes + fallback rows + mask words + ranks +
    scales + q + o."""
    import ctypes

    import torch
    import torch.distributed as dist

    from latticequant_b200 import _lib
    from latticequant_b200 import attention as A
    from latticequant_b200 import sharding as SH
    from latticequant_b200.llm.fused_triton_merge import compress_compact

    lo, hi = SH.sequence_slice(A_S, world, rank, 64)
    S = hi - lo
    k = attention_kv(dev, 4000 + 2 * rank, S)
    kc, _ = compress_compact(k, 4)
    del k
    v = attention_kv(dev, 4001 + 2 * rank, S)
    vc, _ = compress_compact(v, 4)
    del v
    q = attention_query(dev)
    rows = A_B * A_HKV * A_G
    kv, vv = A.compact_view(kc), A.compact_view(vc)
    ws = torch.empty(int(_lib.lib().lq_attn_compact_workspace(A_B * A_HKV, S, A_G, A_D)), dtype=torch.uint8,
                     device=dev)
    o = torch.empty(rows, A_D, dtype=torch.float32 if world > 1 else torch.bfloat16, device=dev)
    lse = torch.empty(rows, dtype=torch.float32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    P = _lib.ptr
    st = torch.cuda.current_stream(dev)

    def step():
        rc = _lib.lib().lq_attn_decode_compact(ctypes.byref(kv), ctypes.byref(vv), P(q), _lib.LQ_BF16, A_B, A_HKV, S,
                                               A_G, A_D, 1 / A_D ** 0.5, P(o), _lib.dtype_code(o.dtype), P(lse),
                                               P(ws), ws.numel(), P(err), _lib.stream_handle(dev))
        if rc != 0:
            raise RuntimeError(f"lq_attn_decode_compact returned {rc}")

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    if int(err.item()):
        raise RuntimeError(f"compact attention error flags {int(err.item()):#x}")
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    words, rank_t = A.compact_index(kc)
    words_v, rank_v = A.compact_index(vc)
    nbytes = (kc.packed.numel() + vc.packed.numel() + 2 * (kc.fallback.numel() + vc.fallback.numel())
              + 4 * (words.numel() + rank_t.numel() + words_v.numel() + rank_v.numel())
              + 4 * (kc.scales.numel() + vc.scales.numel()) + q.numel() * 2 + rows * A_D * o.element_size())
    vals = torch.tensor([ms, float(nbytes), kc.oor_rate + vc.oor_rate], dtype=torch.float64, device=dev)
    if world > 1:
        mx, sm = vals[:1].clone(), vals[1:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, sm])
    ms, tot_bytes, oor2 = vals.tolist()
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    gbps = tot_bytes / (ms * 1e-3) / 1e9
    return {"metric": A_METRIC, "value": gbps, "unit": "GB/s", "ms_per_step": ms,
            "layout": "compact fixed-rate, 4 bits: 4-byte codes + fp16 fallback rows "
                      "(llm/fused_triton_merge.py format)",
            "fallback_share": oor2 / (2 * world), "bytes_per_step_GB": tot_bytes / 1e9,
            "roofline": {"bound": "hbm", "kernel": "attn_compact_mma_kernel + attn_combine_kernel",
                         "achieved": gbps / world, "peak": peak, "unit": "GB/s per GPU",
                         "frac": gbps / world / peak, "peak_kind": peak_kind,
                         "traffic": tot_bytes / world * COMPACT_TRAFFIC_PER_ALG_BYTE / 1e9,
                         "traffic_unit": "GB per launch", "algorithmic_GB": tot_bytes / world / 1e9},
            "gpu_launches": steps * 2}


def bench_config4(dev, rank, world, steps, barrier):
    """Config 4 on `world` ranks: (layer, KV head) units round-robin; the
    rank's K (and V) chunks of each bit rate are coded as ONE batch by one
    Codec, with no host synchronisation inside the timed encode; then decode-
    attention steps over every owned layer."""
    import torch
    import torch.distributed as dist

    from latticequant_b200 import attention as A
    from latticequant_b200 import codec as C
    from latticequant_b200 import sharding as SH

    bits = c4_bits()
    units = SH.shard_units(C4_LAYERS, C4_KV, world, rank)
    layers = {}
    for l, h in units:
        layers.setdefault(l, []).append(h)
    heads_per_layer = {len(hs) for hs in layers.values()}
    if len(heads_per_layer) != 1:
        raise RuntimeError("config 4: ranks must own the same number of heads in every owned layer")
    hr = heads_per_layer.pop()
    shape = (C4_B, hr, C4_S, C4_D)
    bph = C4_S * C4_D // 8
    st = torch.cuda.current_stream(dev)
    bpt = C.blocks_per_token(C4_D, TILE, bph)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    enc_ms, blocks, comp, meta, n_out = 0.0, 0, 0, 0, 0
    per_layer = {}
    # groups of equal bit rate and kind (K: Student-t, V: Gaussian), one after
    # another so only one group's input and buffers are resident; each group's
    # encode is timed on its own (no host synchronisation inside) and the
    # times are summed
    for b in sorted(set(bits[l] for l in layers)):
        ls = [l for l in sorted(layers) if bits[l] == b]
        for kind, student, base in (("K", True, 5000), ("V", False, 9000)):
            x = torch.empty((len(ls),) + shape, dtype=torch.bfloat16, device=dev)
            for i, l in enumerate(ls):
                x[i] = torch.cat([c4_tensor(dev, base + 16 * l + h, 1, student) for h in layers[l]], 1)
            cd = C.Codec(C.Geometry(len(ls), C4_B * hr, bph, TILE), dev)
            # does the group need the outlier side channel (alphabet over L)?
            # decided by an untimed pass, as codec.compress decides it per chunk
            cd.scales(x, b)
            cd.quantize(x)
            cd.build_tables()
            outliers = bool(cd.read_err() & (C._lib.EF_ALPHABET | C._lib.EF_SYMRANGE | C._lib.EF_NOCONVERGE))

            def encode():
                cd.scales(x, b)
                if outliers:
                    cd.quantize_outliers(x, None, bpt)
                else:
                    cd.quantize(x)
                cd.build_tables()
                cd.expand_tables(enc=True, dec=False)
                cd.entropy_encode()

            encode()  # warm-up
            torch.cuda.synchronize()
            cd.err.zero_()
            barrier()
            e0.record(st)
            encode()
            e1.record(st)
            torch.cuda.synchronize()
            enc_ms += e0.elapsed_time(e1)
            C._lib.raise_flags(cd.read_err(), f"config 4 encode ({kind}, {b} bits)")
            for l, ch in zip(ls, cd.chunks(b, shape, torch.bfloat16, outliers)):
                per_layer.setdefault(l, {})[kind] = ch
                blocks += ch.geom.n_vectors
                comp += ch.compressed_bytes()
                meta += ch.metadata_bytes()
                n_out += ch.n_outliers
            del x, cd
            torch.cuda.empty_cache()
    chunks = [(l, hr, A.DecodeAttention(per_layer[l]["K"], per_layer[l]["V"], C4_G)) for l in sorted(per_layer)]
    g = torch.Generator(device=dev)
    g.manual_seed(6006)
    qs = {l: (torch.randn(C4_B, nh * C4_G, C4_D, generator=g, device=dev) / C4_D ** 0.5).to(torch.bfloat16)
          for l, nh, _ in chunks}
    outs = {l: torch.empty(C4_B, nh * C4_G, C4_D, dtype=torch.bfloat16, device=dev) for l, nh, _ in chunks}

    def step():
        for l, nh, op in chunks:
            op(qs[l], outs[l])

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    for _, _, op in chunks:
        if op.flags():
            raise RuntimeError(f"config-4 attention error flags {op.flags():#x}")
    barrier()
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    torch.cuda.synchronize()
    att_ms = e0.elapsed_time(e1) / steps
    vals = torch.tensor([enc_ms, att_ms, float(blocks), float(comp), float(meta), float(n_out)], dtype=torch.float64,
                        device=dev)
    if world > 1:
        mx, sm = vals[:2].clone(), vals[2:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        vals = torch.cat([mx, sm])
    enc_ms, att_ms, blocks, comp, meta, n_out = vals.tolist()
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    att_bytes = comp + meta + 2 * 2 * C4_B * C4_LAYERS * C4_KV * C4_G * C4_D
    enc_alg = blocks * 16.0 + comp
    return {"workload": "config4: Qwen2.5-7B KV 28L x 4 kv-heads x D128, B4, ctx 131072, bits per layer "
                        f"{bits} (K Student-t(3), V N(0,1))",
            "parallelism": f"(layer, kv-head) units round-robin over {world} ranks, no collective",
            "encode": {"metric": "E8+rANS encode Gvec/s", "value": blocks / (enc_ms * 1e-3) / 1e9, "unit": "Gvec/s",
                       "ms": enc_ms, "note": "whole model: per rank one Codec batch per (bit rate, K/V), each "
                                             "timed without host synchronisation inside, times summed",
                       "roofline": {"bound": "hbm", "achieved": enc_alg / (enc_ms * 1e-3) / 1e9 / world,
                                    "peak": peak, "unit": "GB/s per GPU",
                                    "frac": enc_alg / (enc_ms * 1e-3) / 1e9 / world / peak, "peak_kind": peak_kind,
                                    "algorithmic": "bf16 in + compressed out"}},
            "attention": {"metric": A_METRIC, "value": att_bytes / (att_ms * 1e-3) / 1e9, "unit": "GB/s",
                          "ms_per_step": att_ms, "tokens_per_s": C4_B * 1e3 / att_ms,
                          "roofline": {"bound": "hbm", "achieved": att_bytes / (att_ms * 1e-3) / 1e9 / world,
                                       "peak": peak, "unit": "GB/s per GPU",
                                       "frac": att_bytes / (att_ms * 1e-3) / 1e9 / world / peak,
                                       "peak_kind": peak_kind}},
            "bits_per_dim": comp * 8 / (blocks * 8), "outlier_records": int(n_out),
            "gpu_launches": steps * 3 * len(chunks) * world}


C1_VEC, C1_D = 262144, 128


def c1_input(dev, seed):
    """Config 1: (262144, 128) fp32, N(0,1) times a log-normal(0, 0.5) magnitude per vector."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(C1_VEC, C1_D, generator=g, device=dev) *
            torch.exp(0.5 * torch.randn(C1_VEC, 1, generator=g, device=dev))).contiguous()


def bench_config1(dev, rank, world, steps, warmup, barrier, with_oracle):
    """Config 1 per rank (weak scaling): one chunk of 262,144 heads x 16 blocks
    (a per-vector fp16 scale), encode + decode to fp32 per step, CUDA-graphed;
    reconstructed MSE and bitstream bytes, checked against the C oracle's for
    the same input when `with_oracle` (rank 0 only)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from latticequant_b200 import codec as C

    x = c1_input(dev, 7100 + rank)
    bph = C1_D // 8
    n_blocks = C1_VEC * bph
    cd = C.Codec(C.Geometry(1, C1_VEC, bph, TILE), dev)
    out = torch.empty(n_blocks * 8, dtype=torch.float32, device=dev)

    def step():
        cd.encode(x, BITS)
        cd.expand_tables(enc=False, dec=True)
        cd.decode(out)

    step()
    torch.cuda.synchronize()
    if cd.read_err():
        raise RuntimeError(f"config 1: device error flags {cd.read_err():#x}")
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graph
    n_words = cd.n_words()
    comp = 4 * n_words + (n_blocks + 7) // 8 + 2 * C1_VEC
    lanes = C.Geometry(1, C1_VEC, bph, TILE).n_lanes
    meta = 8 * lanes
    diff = out.view(C1_VEC, C1_D).double() - x.double()
    mse = float((diff * diff).mean())
    nmse = mse / float((x.double() ** 2).mean())

    # e2e through the same calls with host buffers: x in, decoded vectors out
    host_x = x.cpu().pin_memory()
    host_out = torch.empty(n_blocks * 8, dtype=torch.float32).pin_memory()
    dx = torch.empty_like(x)

    def e2e_step():
        dx.copy_(host_x, non_blocking=True)
        cd.encode(dx, BITS)
        cd.expand_tables(enc=False, dec=True)
        cd.decode(out)
        host_out.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    k2 = max(2, min(steps, 5))
    e0.record(st)
    for _ in range(k2):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1) / k2
    vals = torch.tensor([ms, ems], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, ems = vals.tolist()
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    alg = n_blocks * (32.0 + 2 * comp / n_blocks + 32.0)  # fp32 in, compressed out, compressed in, fp32 out
    res = {"metric": "E8+rANS encode/decode Gvec/s", "value": world * n_blocks / (ms * 1e-3) / 1e9,
           "unit": "Gvec/s", "ms_per_step": ms,
           "workload": "config1: 262,144 x 128 fp32 (N(0,1) x lognormal(0,0.5) per vector), per-vector fp16 "
                       "scale (one chunk of 262,144 heads x 16 blocks), 4 b/dim, encode + decode to fp32",
           "mse": mse, "nmse": nmse, "bitstream_bytes": comp, "bits_per_dim": comp * 8 / (n_blocks * 8),
           "bytes_rule": "4 x words + coset bits + 2 B per scale (llm/compressed_kv_cache.py:113-119)",
           "lane_metadata_bytes": meta,
           "step_roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": alg / (ms * 1e-3) / 1e9 / peak, "peak_kind": peak_kind,
                             "algorithmic_GB": alg / 1e9},
           "e2e": {"value": world * n_blocks / (ems * 1e-3) / 1e9, "unit": "Gvec/s", "ms_per_step": ems,
                   "h2d_bytes_per_step": x.numel() * 4, "d2h_bytes_per_step": out.numel() * 4},
           "gpu_launches": steps * 10}
    if with_oracle:
        try:
            import oracle.lq_oracle as O

            O.build()
            xn = x.cpu().numpy()
            t0 = time.perf_counter()
            ref = O.compress_chunk(xn, O.DT_F32, C1_VEC, bph, BITS, tile_blocks=TILE, ties="stable")
            rec = O.decompress_chunk(ref, O.DT_F32).reshape(C1_VEC, C1_D)
            dt = time.perf_counter() - t0
            r_bytes = 4 * int(ref.words.size) + (n_blocks + 7) // 8 + 2 * C1_VEC
            d = rec.astype(np.float64) - xn.astype(np.float64)
            r_mse = float((d * d).mean())
            same = (int(ref.words.size) == n_words and
                    np.array_equal(ref.words, cd.words[:n_words].cpu().numpy().view(np.uint32)) and
                    np.array_equal(rec.reshape(-1).view(np.uint32), out.cpu().numpy().view(np.uint32)))
            # the reference's own layout: one 16-stream chunk, numpy table ties,
            # plus the one spare word per stream the reference stores
            refl = O.compress_chunk(xn, O.DT_F32, C1_VEC, bph, BITS, tile_blocks=None, ties="numpy")
            n0 = int(refl.tile_n0.sum())
            n_streams = 8 * (n0 > 0) + 8 * (n_blocks - n0 > 0)  # an empty coset has no streams
            rl_bytes = 4 * (int(refl.words.size) + n_streams) + (n_blocks + 7) // 8 + 2 * C1_VEC
            res["oracle"] = {"mse": r_mse, "bitstream_bytes": r_bytes, "identical_words_and_decode": bool(same),
                             "mse_equal": r_mse == mse, "bytes_equal": r_bytes == comp,
                             "reference_layout_bytes": rl_bytes,
                             "reference_layout_bits_per_dim": rl_bytes * 8 / (n_blocks * 8),
                             "note": "C oracle (oracle/lq_oracle_codec.c) on the same input: same lane layout "
                                     "(1024-block tiles) and stable table ties; reference_layout_* = one "
                                     "16-stream chunk as the reference codes it (numpy ties, spare word per "
                                     f"stream); oracle time {dt:.1f} s"}
        except Exception as e:  # the comparison is reported, not required
            res["oracle"] = {"unavailable": str(e)[:200]}
    return res


C5_METRIC = "decode tok/s"


def bench_config5(dev, rank, world, args, barrier):
    """a random-init Llama-3.1-8B-architecture model (bf16
    weights N(0, 0.02), replicated on every rank) decoding through
    CompressedAttentionKVCache at 4 bits/dim: prefill of seeded random ids,
    then greedy tokens, each decode step attending over the compressed cache
    with the fused kernels.  At N > 1 the cache is sharded by KV head
    (sharding.head_slice); every layer all-gathers the heads' outputs.  The
    timed region covers the decode steps after `warmup` of them, including a
    per-step copy of the new token ids to pinned host memory."""
    import time

    import torch
    import torch.distributed as dist
    from transformers import LlamaConfig, LlamaForCausalLM

    from latticequant_b200 import sharding as SH
    from latticequant_b200.llm.compressed_attention import CompressedAttentionKVCache
    from latticequant_b200.llm.graph_decode import GraphedDecodeStep

    L, B, P, T, W = args.c5_layers, args.c5_batch, args.c5_prefill, args.c5_gen, args.warmup
    if T <= W:
        raise ValueError("--c5-gen must exceed --warmup")
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=L,
                      num_attention_heads=32, num_key_value_heads=8, max_position_embeddings=131072,
                      rope_theta=500000.0, initializer_range=0.02, rms_norm_eps=1e-5, tie_word_embeddings=False)
    torch.manual_seed(5005)  # the same weights on every rank
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = LlamaForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    model.eval()
    g = torch.Generator(device=dev)
    g.manual_seed(5006)
    ids = torch.randint(0, cfg.vocab_size, (B, P), generator=g, device=dev)
    hr = SH.head_slice(cfg.num_key_value_heads, world, rank) if world > 1 else None
    cache = CompressedAttentionKVCache(4, tail_tokens=args.c5_tail, head_range=hr, layout=args.c5_layout).bind(model)
    host = torch.empty(T, B, dtype=torch.int64, pin_memory=True)
    st = torch.cuda.current_stream(dev)
    e_dec0, e_dec1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        barrier()
        torch.cuda.synchronize()
        t0 = time.time()
        out = model(ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        del out
        torch.cuda.synchronize()
        prefill_s = time.time() - t0
        stepper = None if args.c5_eager else GraphedDecodeStep(model, cache)
        for i in range(T):
            if i == W:
                barrier()
                torch.cuda.synchronize()
                e_dec0.record(st)
            if stepper is not None:
                nxt = stepper.step(nxt)
            else:
                out = model(nxt, past_key_values=cache, use_cache=True)
                nxt = out.logits[:, -1].argmax(-1, keepdim=True)
                del out
            host[i].copy_(nxt.view(-1), non_blocking=True)
        e_dec1.record(st)
        torch.cuda.synchronize()
        captures = stepper.captures if stepper is not None else 0
        capture_s = stepper.capture_s if stepper is not None else 0.0
        if stepper is not None:
            stepper.release()  # the graph holds collectives when sharded: gone before the process group
        # the attention of one layer (every compressed part, the exact tail and
        # the LSE merge), timed eagerly after the run, and the fused kernel over
        # the layer's prefill chunk alone (its roofline)
        Hq = cfg.num_attention_heads // world
        G = cfg.num_attention_heads // cfg.num_key_value_heads
        D = cfg.hidden_size // cfg.num_attention_heads
        gq = torch.Generator(device=dev)
        gq.manual_seed(5007)
        q4 = (torch.randn(B, Hq, 1, D, generator=gq, device=dev) / D ** 0.5).to(torch.bfloat16)
        reps = 10
        for _ in range(2):
            cache.decode_attention(0, q4)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(reps):
            cache.decode_attention(0, q4)
        e1.record(st)
        torch.cuda.synchronize()
        layer_attn_ms = e0.elapsed_time(e1) / reps
        part = cache._state[0].parts[0]
        op = part.op(G)
        q3 = q4.view(B, Hq, D)
        o3 = torch.empty(B, Hq, D, dtype=torch.float32, device=dev)
        l3 = torch.empty(B, Hq, dtype=torch.float32, device=dev)
        for _ in range(2):
            op(q3, o3, l3)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(reps):
            op(q3, o3, l3)
        e1.record(st)
        torch.cuda.synchronize()
        kern_ms = e0.elapsed_time(e1) / reps
        if part.layout == "compact":
            kern_bytes = compact_chunk_bytes(part.k) + compact_chunk_bytes(part.v)
        else:
            kern_bytes = (part.k.compressed_bytes() + part.v.compressed_bytes() + part.k.metadata_bytes() +
                          part.v.metadata_bytes())
        kern_bytes += q3.numel() * 2 + o3.numel() * 4
    vals = torch.tensor([e_dec0.elapsed_time(e_dec1), layer_attn_ms, kern_ms],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, layer_attn_ms, kern_ms = vals.tolist()
    flags = cache.flags()
    if flags:
        raise RuntimeError(f"config-5 attention error flags {flags:#x}")
    steps = T - W
    comp = sum(l.total_bytes for l in cache._comp_keys + cache._comp_values if l is not None)
    mem = torch.cuda.max_memory_allocated(dev)
    if rank != 0:
        return None
    peak, peak_kind = measured_peaks()
    return {"metric": C5_METRIC, "value": B * steps * 1e3 / ms, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": W, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16", "data": "synthetic (random-init weights N(0,0.02), seeded random token ids)",
            "config": {"workload": f"config5: Llama-3.1-8B architecture ({L} layers, 4096 hidden, 32 q / 8 kv heads), "
                                   f"batch {B}, prefill {P} random ids, {T} generated tokens, 4 b/dim KV "
                                   f"({'rANS lanes' if args.c5_layout == 'rans' else 'compact fixed-rate layout'}; "
                                   f"decode tokens encoded every {args.c5_tail})",
                       "parallelism": f"KV-head-sharded cache over {world} GPUs (weights replicated, per-layer "
                                      "all-gather of attention heads)" if world > 1 else "single GPU",
                       "global_batch": B, "seq_len": P + T},
            "decode": "eager" if args.c5_eager else f"CUDA graph replays ({captures} captures; a tail flush "
                                                     "that replaces a buffer the step reads is followed by a "
                                                     "new capture, inside the timed region)",
            "capture_s": capture_s,
            "prefill_s": prefill_s, "compressed_cache_GB_rank0": comp / 1e9,
            "max_memory_GB_rank0": mem / 1e9,
            "attention": {"layer_ms": layer_attn_ms, "share_of_step": L * layer_attn_ms / (ms / steps),
                          "note": "one layer's attention (compressed parts + exact tail + merge) timed eagerly "
                                  "after the run, x layers / step time",
                          "roofline": {"bound": "hbm", "kernel": "fused attention over a layer's prefill chunk "
                                                                 f"({part.layout} layout)",
                                       "kernel_ms": kern_ms, "achieved": kern_bytes / (kern_ms * 1e-3) / 1e9,
                                       "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                                       "frac": kern_bytes / (kern_ms * 1e-3) / 1e9 / peak,
                                       "algorithmic_GB": kern_bytes / 1e9}},
            "e2e": {"value": B * steps * 1e3 / ms, "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                    "d2h_bytes_per_step": B * 8,
                    "note": "decode steps with the token ids copied to pinned host memory each step"}}


def run_reference(args):
    """--impl reference: the reference's CPU path (C oracle port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n_thr = os.cpu_count() or 1
    sample = max(2, min(N_CHUNKS, 2 * n_thr))
    for _ in range(args.warmup):
        cpu_baseline(n_thr, sample_chunks=2)
    vals = []
    for _ in range(args.steps):
        v, blocks, dt = cpu_baseline(n_thr, sample_chunks=sample)
        vals.append(v)
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": BLOCKS / (v * 1e9) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded config-2 K/V)",
            "config": {"workload": "config2: Llama-3.1-8B KV 32Lx8Hx8192x128 bf16, 4 b/dim, encode+decode",
                       "global_batch": 1, "seq_len": SEQ, "parallelism": "host threads",
                       "l2": "inputs larger than L2"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": n_thr, "kind": "port",
                             "sample": f"{sample} of 64 chunks per step (oracle/lq_oracle_codec.c, pthreads)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_attn:
        va, nb, dt = cpu_attention_baseline()
        line["attention"] = {"metric": A_METRIC, "value": va, "unit": "GB/s",
                             "cpu_baseline": {"value": va, "unit": "GB/s", "cores": 1, "kind": "port",
                                              "sample": f"1 of {A_B} batch rows, 2048 tokens ({nb} B, {dt:.2f} s)"}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-attn", action="store_true", help="skip the config-3 attention measurement")
    ap.add_argument("--e2e-group", type=int, default=E2E_GROUP, help="chunks per pipelined e2e transfer group")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-4 mixed-rate measurement")
    ap.add_argument("--no-c1", action="store_true", help="skip the config-1 measurement")
    ap.add_argument("--no-c5", action="store_true", help="skip the config-5 decode measurement")
    ap.add_argument("--no-c5-compact", action="store_true",
                    help="skip the second config-5 run with the compact-layout cache")
    ap.add_argument("--only-c5", action="store_true",
                    help="run only config 5 (Llama-3.1-8B-shaped decode through the compressed cache) and print its line")
    ap.add_argument("--c5-layers", type=int, default=32)
    ap.add_argument("--c5-batch", type=int, default=32)
    ap.add_argument("--c5-prefill", type=int, default=16384)
    ap.add_argument("--c5-gen", type=int, default=256)
    ap.add_argument("--c5-eager", action="store_true", help="config 5 decode steps run eagerly (no CUDA graph)")
    ap.add_argument("--c5-tail", type=int, default=64, help="decode tokens encoded together (the cache's tail_tokens)")
    ap.add_argument("--c5-layout", default="rans", choices=["rans", "compact"],
                    help="cache layout of config 5: entropy-coded lanes or the compact fixed-rate layout")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="layers of the cache (profiling runs use fewer; bench lines use 32)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from latticequant_b200 import codec as C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.only_c5:
        line = bench_config5(dev, rank, world, args, barrier)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    global N_CHUNKS, BLOCKS
    N_CHUNKS = 2 * args.layers
    BLOCKS = N_CHUNKS * N_KV * BPH
    x = make_cache(dev, rank, args.layers)
    geom = C.Geometry(N_CHUNKS, N_KV, BPH, TILE)
    cd = C.Codec(geom, dev)
    out = torch.empty(BLOCKS * 8, dtype=torch.bfloat16, device=dev)

    def step():
        cd.encode(x, BITS)
        cd.expand_tables(enc=False, dec=True)
        cd.decode(out)

    # launches per step: scales 1-2, quantize 1, tables 2 (+1 expand dec), encode 5, decode 1
    launches_per_step = (1 if C.lib().lq_head_scales_workspace(N_CHUNKS * N_KV, BPH * 8) == 0 else 2) + 1 + 2 + 5 + 1 + 1

    # correctness gate: one eager step, error word clear, lossless round trip on a sample chunk
    step()
    torch.cuda.synchronize()
    if cd.read_err():
        raise RuntimeError(f"device error flags {cd.read_err():#x}")

    graph = None
    if not args.no_graph:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()

    def run():
        if graph is not None:
            graph.replay()
        else:
            step()

    for _ in range(max(args.warmup, 3)):
        run()
    torch.cuda.synchronize()

    # phase timing (eager, CUDA events on the launching stream) for the roofline
    st = torch.cuda.current_stream(dev)
    names = ["scales", "quantize", "tables", "encode", "expand_dec", "decode"]
    acc = {n: 0.0 for n in names}
    reps = 3
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        ev[0].record(st)
        cd.scales(x, BITS); ev[1].record(st)
        cd.quantize(x); ev[2].record(st)
        cd.build_tables(); cd.expand_tables(enc=True, dec=False); ev[3].record(st)
        cd.entropy_encode(); ev[4].record(st)
        cd.expand_tables(enc=False, dec=True); ev[5].record(st)
        cd.decode(out); ev[6].record(st)
        torch.cuda.synchronize()
        for i, n in enumerate(names):
            acc[n] += ev[i].elapsed_time(ev[i + 1]) / reps
    n_words = cd.n_words()
    comp_bytes = 4 * n_words + N_CHUNKS * ((N_KV * BPH + 7) // 8) + 2 * N_CHUNKS * N_KV

    # timed region
    sampler = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        run()
    e1.record(st)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * BLOCKS / (ms * 1e-3) / 1e9

    # e2e through the public API with host buffers: the cache goes host -> device,
    # is encoded and decoded, and the decoded cache comes back, in groups of
    # E2E_GROUP chunks on three streams so the two PCIe directions and the codec
    # overlap (copy-in of group g+1 and copy-out of group g-1 under the coding of g)
    e2e = None
    if not args.no_e2e:
        grp = args.e2e_group if args.e2e_group > 0 and N_CHUNKS % args.e2e_group == 0 else N_CHUNKS
        n_grp = N_CHUNKS // grp
        host_x = x.cpu().pin_memory()
        host_out = torch.empty(BLOCKS * 8, dtype=torch.bfloat16).pin_memory()
        dx = torch.empty_like(x)
        cg = C.Codec(C.Geometry(grp, N_KV, BPH, TILE), dev)
        s_in, s_code, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        per = grp * N_KV * BPH * 8
        ev_in = [torch.cuda.Event() for _ in range(n_grp)]
        ev_code = [torch.cuda.Event() for _ in range(n_grp)]

        def e2e_step():
            for g in range(n_grp):
                with torch.cuda.stream(s_in):
                    dx[g * grp:(g + 1) * grp].copy_(host_x[g * grp:(g + 1) * grp], non_blocking=True)
                    ev_in[g].record(s_in)
                with torch.cuda.stream(s_code):
                    s_code.wait_event(ev_in[g])
                    cg.encode(dx[g * grp:(g + 1) * grp], BITS)
                    cg.expand_tables(enc=False, dec=True)
                    cg.decode(out[g * per:(g + 1) * per])
                    ev_code[g].record(s_code)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_code[g])
                    host_out[g * per:(g + 1) * per].copy_(out[g * per:(g + 1) * per], non_blocking=True)
            st.wait_stream(s_out)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if cg.read_err():
            raise RuntimeError(f"device error flags {cg.read_err():#x}")
        barrier()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        k2 = max(2, min(args.steps, 5))
        f0.record(st)
        s_in.wait_stream(st)
        for _ in range(k2):
            e2e_step()
            s_in.wait_stream(st)
        f1.record(st)
        torch.cuda.synchronize()
        ems = f0.elapsed_time(f1) / k2
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        # the round trip must reproduce the device-resident result
        if not torch.equal(host_out[:per].to(dev).view(torch.int16), out[:per].view(torch.int16)):
            raise RuntimeError("e2e output differs from the device result")
        e2e = {"value": world * BLOCKS / (ems * 1e-3) / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
               "ms_per_step": ems, "pipeline": f"{n_grp} groups of {grp} chunks, 3 streams"}

    # roofline of each phase on its OWN algorithmic bytes (what that phase must
    # move at the least): scales read the bf16 input; quantize reads it and
    # writes the coset bits; the lane encoder writes the words; decode reads
    # words + coset bits + scales and writes bf16.  The symbol columns between
    # quantize and the encoder are an intermediate and count nowhere.
    peak, peak_kind = measured_peaks()
    comp_per_block = comp_bytes / BLOCKS
    words_per_block = 4.0 * n_words / BLOCKS
    alg = {"scales": BLOCKS * 16.0, "quantize": BLOCKS * (16.0 + 1.0 / 8), "tables": 0.0,
           "encode": BLOCKS * words_per_block, "expand_dec": 0.0, "decode": BLOCKS * (comp_per_block + 16.0)}
    dom = max(names, key=lambda n: acc[n])
    achieved = alg[dom] / (acc[dom] * 1e-3) / 1e9
    phases = {n: {"ms": round(acc[n], 4), "algorithmic_GB": alg[n] / 1e9,
                  "frac": (alg[n] / (acc[n] * 1e-3) / 1e9 / peak) if alg[n] and acc[n] else None}
              for n in names}
    step_alg = BLOCKS * (16.0 + comp_per_block) + BLOCKS * (comp_per_block + 16.0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_thr = os.cpu_count() or 1
        n_smp = max(2, min(N_CHUNKS, n_thr))  # one chunk per host thread (the port threads over chunks)
        v, blocks, dt = cpu_baseline(n_thr, sample_chunks=n_smp, min_seconds=10.0)
        cpu = {"value": v, "unit": UNIT, "cores": n_thr, "kind": "port",
               "sample": f"{blocks} blocks ({n_smp} config-2 chunks coded and decoded "
                         f"{blocks // (n_smp * N_KV * BPH)} times), oracle/lq_oracle_codec.c on "
                         f"{n_thr} threads, {dt:.1f} s"}

    attn = None
    if not args.no_attn:
        del x, out
        cd = None
        torch.cuda.empty_cache()
        attn = bench_attention(dev, rank, world, args.steps, args.warmup, barrier)
        torch.cuda.empty_cache()
        attn_c = bench_attention_compact(dev, rank, world, args.steps, args.warmup, barrier)
        if rank == 0:
            attn["compact_layout"] = attn_c
    c4 = None
    if not args.no_c4:
        torch.cuda.empty_cache()
        c4 = bench_config4(dev, rank, world, max(2, min(args.steps, 5)), barrier)
    c1 = None
    if not args.no_c1:
        torch.cuda.empty_cache()
        c1 = bench_config1(dev, rank, world, args.steps, args.warmup, barrier, with_oracle=world == 1 and rank == 0)
    c5 = None
    if not args.no_c5:
        torch.cuda.empty_cache()
        c5 = bench_config5(dev, rank, world, args, barrier)
        if not args.no_c5_compact and args.c5_layout == "rans":
            torch.cuda.empty_cache()
            args.c5_layout = "compact"
            c5c = bench_config5(dev, rank, world, args, barrier)
            args.c5_layout = "rans"
            if rank == 0:
                c5["compact_layout"] = c5c

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded config-2 K/V)",
                "config": {"workload": f"config2: Llama-3.1-8B KV {args.layers}Lx8Hx8192x128 bf16, 4 b/dim, "
                                       "encode+decode",
                           "global_batch": world, "seq_len": SEQ, "parallelism": f"dp{world} (chunks per rank)",
                           "tile_blocks": TILE, "l2": "inputs larger than L2 (1 GiB per rank)",
                           "cuda_graph": graph is not None},
                "bits_per_dim": comp_bytes * 8 / (BLOCKS * 8),
                "phase_ms": {n: round(acc[n], 4) for n in names},
                "phases": phases,
                "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_kind": peak_kind,
                             "traffic": (TRAFFIC_PER_BLOCK[dom] * BLOCKS / 1e9) if dom in TRAFFIC_PER_BLOCK else None,
                             "traffic_unit": "GB per launch", "algorithmic_GB": alg[dom] / 1e9},
                "step_roofline": {"bound": "hbm", "achieved": step_alg / (ms * 1e-3) / 1e9, "peak": peak,
                                  "unit": "GB/s per GPU", "frac": step_alg / (ms * 1e-3) / 1e9 / peak,
                                  "peak_kind": peak_kind, "algorithmic_GB": step_alg / 1e9,
                                  "algorithmic": "bf16 in + compressed out (encode), compressed in + bf16 out "
                                                 "(decode)"},
                "clocks": clocks, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
                "cpu_baseline": cpu, "attention": attn, "config4": c4, "config1": c1, "config5": c5}
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
