"""Rate of the reference's own Python compression path on this host's cores.

Test infrastructure, not part of the product: it imports the reference's
`CompressedKVCache._compress_tensor` (llm/compressed_kv_cache.py:176-257,
torch E8 search + numpy table build + the Python rANS loop of
core/gpu_ans.py) from a checkout named by LQ_REFERENCE (required) and times
it on config-2-shaped chunks (8 KV heads x S tokens x 128, bf16, 4 b/dim),
first in one process, then in a pool of P processes (spawned, each coding
its own chunk at once).  A GPU box has no reference checkout; this runs
where one is.

    LQ_REFERENCE=<checkout> python oracle/time_reference_python.py [--tokens S] [--procs P]

Prints one JSON line: blocks/s for one process and for the pool.
"""
import argparse
import json
import multiprocessing as mp
import os
import sys
import time


def _setup():
    ref = os.environ.get("LQ_REFERENCE")
    if not ref or not os.path.isdir(ref):
        sys.exit("time_reference_python.py: set LQ_REFERENCE to the reference checkout")
    for sub in ("core", "llm"):
        p = os.path.join(ref, sub)
        if p not in sys.path:
            sys.path.insert(0, p)


def _code_one(args):
    """Code one seeded chunk; returns (blocks, seconds)."""
    seed, tokens = args
    _setup()
    import torch

    torch.set_num_threads(1)
    import compressed_kv_cache as ref_kv

    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(1, 8, tokens, 128, generator=g) *
         torch.exp(0.5 * torch.randn(1, 8, tokens, 1, generator=g))).to(torch.bfloat16)
    cache = ref_kv.CompressedKVCache(bits_per_dim=4)
    t0 = time.perf_counter()
    cache._compress_tensor(x)
    return x.numel() // 8, time.perf_counter() - t0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=1024, help="tokens per chunk (8 heads x tokens x 128)")
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    _setup()
    nb, dt = _code_one((1, args.tokens))
    ctx = mp.get_context("spawn")
    with ctx.Pool(args.procs) as pool:
        pool.map(_code_one, [(100 + i, 64) for i in range(args.procs)])  # imports and warm-up in every worker
        t0 = time.perf_counter()
        res = pool.map(_code_one, [(200 + i, args.tokens) for i in range(args.procs)])
        wall = time.perf_counter() - t0
    total = sum(r[0] for r in res)
    print(json.dumps({"path": "CompressedKVCache._compress_tensor (llm/compressed_kv_cache.py:176-257), 4 b/dim",
                      "chunk": f"1 x 8 x {args.tokens} x 128 bf16", "one_process_blocks_per_s": nb / dt,
                      "one_process_s": dt, "pool_procs": args.procs, "pool_blocks_per_s": total / wall,
                      "pool_wall_s": wall, "host_cores": os.cpu_count()}))


if __name__ == "__main__":
    main()
