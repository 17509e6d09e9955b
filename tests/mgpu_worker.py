"""One rank of tests/test_multi_gpu.py (launched by torch.distributed.run, one
process per GPU, NCCL).  Every rank builds the same seeded rows, samples its
column shard through verbo_b200.sharded (shard top-k -> NCCL all-gather ->
merge), and rank 0 checks the ids against the unsharded CUDA path on the full
rows; every rank checks that all ranks drew the same ids.  Then the
tensor-parallel logits tail: each rank holds a vocab shard of a seeded Q8 head,
turns the same hidden rows into its shard's logits and picks through the same
sharded merge; rank 0 checks the ids against the full head's tail on one GPU
followed by the unsharded pick.  Exit status 0 on success."""
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
from verbo_b200 import sharded  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        rows, V, H = 64, 151936, 256
        g = np.random.default_rng(2024)
        x = (g.standard_normal((rows, V)) * 3).astype(np.float32)
        hist = g.integers(0, V, size=rows * H).astype(np.int32)
        off = np.arange(rows + 1, dtype=np.int64) * H
        opts = vb.Sampling(temp=0.9, top_k=64, top_p=1.0, min_p=0.1, repeat=1.15, repeat_last=H)
        lo, hi = sharded.shard_bounds(V, world, rank)
        shard = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi])).to(dev)
        dh, do = torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev)
        st = np.array(vb.seed_states(list(range(1, rows + 1))), dtype=np.uint64)
        rng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
        ids = [sharded.sample_vocab_sharded(shard, lo, V, opts, 64, rng, dh, do).clone() for _ in range(3)]
        vb.check()
        got = torch.stack(ids)
        every = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(every, got)
        ok = all(torch.equal(e, got) for e in every)
        if rank == 0:
            full = torch.from_numpy(x).to(dev)
            rng2 = torch.from_numpy(st.view(np.int64).copy()).to(dev)
            want = torch.stack([vb.sample(full, opts, rng=rng2, hist=dh, hist_off=do).clone() for _ in range(3)])
            ok = ok and torch.equal(want, got)
            print(f"rank0: sharded over {world} GPUs == unsharded: {torch.equal(want, got)}; ranks agree: "
                  f"{all(torch.equal(e, got) for e in every)}", flush=True)
        # tensor-parallel logits tail: head rows sharded, logits never gathered
        tv, td = 32000, 896
        tg = np.random.default_rng(7)
        tq = tg.integers(-127, 128, size=(tv, td), dtype=np.int8)
        ts = (np.abs(tg.standard_normal((tv, td // 32))) * 0.004 + 1e-4).astype(np.float16).view(np.uint16)
        tn = (1 + 0.1 * tg.standard_normal(td)).astype(np.float32)
        hx = torch.from_numpy((tg.standard_normal((rows, td)) * 3).astype(np.float32)).to(dev)
        tlo, thi = sharded.shard_bounds(tv, world, rank)
        tail = vb.Tail("q8", tq[tlo:thi], ts[tlo:thi], tn, 1e-6, device=dev.index)
        topts = vb.Sampling(temp=0.8, top_k=40, top_p=0.9)
        trng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
        tids = torch.stack([sharded.sample_tail_sharded(tail, hx, tlo, tv, topts, 64, trng).clone()
                            for _ in range(2)])
        vb.check()
        tevery = [torch.empty_like(tids) for _ in range(world)]
        dist.all_gather(tevery, tids)
        ok = ok and all(torch.equal(e, tids) for e in tevery)
        if rank == 0:
            full_tail = vb.Tail("q8", tq, ts, tn, 1e-6, device=dev.index)
            trng2 = torch.from_numpy(st.view(np.int64).copy()).to(dev)
            twant = torch.stack([vb.sample(full_tail.logits(hx), topts, rng=trng2).clone() for _ in range(2)])
            vb.check()
            tok = torch.equal(twant, tids)
            ok = ok and tok
            print(f"rank0: tensor-parallel tail over {world} GPUs == one-GPU tail + pick: {tok}", flush=True)
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        return 0 if flag.item() == 1 else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
