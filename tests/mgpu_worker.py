"""One rank of tests/test_multi_gpu.py (launched by torch.distributed.run, one
process per GPU).  The ranks build the library's own communicator
(verbo_b200.sharded.make_comm: rank 0's NCCL id broadcast through the process
group), every rank builds the same seeded rows, samples its column shard with
verbo_cuda_sharded_sample (shard top-k -> one NCCL all-gather of packed
candidates -> merge), and rank 0 checks the ids of three consecutive picks
against the C oracle (the reference's Sampler::pick restated) on the full
rows; every rank checks that all ranks drew the same ids.  Then the
tensor-parallel logits tail: each rank holds a vocab shard of a seeded Q8 head,
turns the same hidden rows into its shard's logits and picks through the same
communicator; rank 0 checks the ids against the oracle's tail (the reference's
scalar rmsnorm + quant_act + matmul restated) followed by the oracle's pick.
Exit status 0 on success."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import verbo_b200 as vb  # noqa: E402
from oracle import pyoracle as po  # noqa: E402
from tests.gpu_util import compare, run_oracle  # noqa: E402
from verbo_b200 import sharded  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        comm = sharded.make_comm(dev.index)
        rows, V, H = 64, 151936, 256
        g = np.random.default_rng(2024)
        x = (g.standard_normal((rows, V)) * 3).astype(np.float32)
        hist = g.integers(0, V, size=rows * H).astype(np.int32)
        off = np.arange(rows + 1, dtype=np.int64) * H
        kw = dict(temp=0.9, top_k=64, top_p=0.9, min_p=0.1, repeat=1.15, repeat_last=H)
        opts = vb.Sampling(**kw)
        lo, hi = sharded.shard_bounds(V, world, rank)
        shard = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi])).to(dev)
        dh, do = torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev)
        seeds = np.arange(1, rows + 1, dtype=np.uint64)
        st = po.seed_states(seeds)
        rng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
        ids = [sharded.sample_vocab_sharded(comm, shard, lo, V, opts, 64, rng, dh, do).clone() for _ in range(3)]
        comm.wait(timeout_ms=30000)
        vb.check()
        got = torch.stack(ids)
        every = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(every, got)
        agree = all(torch.equal(e, got) for e in every)
        ok = agree
        if rank == 0:
            ora, ost, _ = run_oracle(x, kw, seeds, hist, off, steps=3)
            n = compare(got.cpu().numpy().T, ora, ost, "sharded vs oracle")
            print(f"rank0: sharded over {world} GPUs == oracle: True ({n} boundary rows differ); "
                  f"ranks agree: {agree}", flush=True)
        # tensor-parallel logits tail: head rows sharded, logits never gathered
        tv, td = 32000, 896
        tg = np.random.default_rng(7)
        tq = tg.integers(-127, 128, size=(tv, td), dtype=np.int8)
        ts = (np.abs(tg.standard_normal((tv, td // 32))) * 0.004 + 1e-4).astype(np.float16).view(np.uint16)
        tn = (1 + 0.1 * tg.standard_normal(td)).astype(np.float32)
        hxn = (tg.standard_normal((rows, td)) * 3).astype(np.float32)
        hx = torch.from_numpy(hxn).to(dev)
        tlo, thi = sharded.shard_bounds(tv, world, rank)
        tail = vb.Tail("q8", tq[tlo:thi], ts[tlo:thi], tn, 1e-6, device=dev.index)
        tkw = dict(temp=0.8, top_k=40, top_p=0.9)
        topts = vb.Sampling(**tkw)
        trng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
        tids = torch.stack([sharded.sample_tail_sharded(comm, tail, hx, tlo, tv, topts, 64, trng).clone()
                            for _ in range(2)])
        comm.wait(timeout_ms=30000)
        vb.check()
        tevery = [torch.empty_like(tids) for _ in range(world)]
        dist.all_gather(tevery, tids)
        ok = ok and all(torch.equal(e, tids) for e in tevery)
        if rank == 0:
            lg, _, _ = po.logits_tail("q8", tq, ts, tn, 1e-6, hxn)
            tora, tost, _ = run_oracle(lg, tkw, seeds, steps=2)
            n = compare(tids.cpu().numpy().T, tora, tost, "tensor-parallel tail vs oracle")
            print(f"rank0: tensor-parallel tail over {world} GPUs == oracle tail + pick: True "
                  f"({n} boundary rows differ)", flush=True)
        tail.close()
        comm.close()
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        return 0 if flag.item() == 1 else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
