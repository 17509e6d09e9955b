"""One call of every kernel family of the library, on one GPU, for per-kernel
profiling (a DRAM-throughput table of every kernel from one capture).

    python -m verbo_b200.kernel_tour

Steps, each a public call of the library on seeded synthetic inputs with the
benchmark configurations' options (verbo_b200/workloads.py), sized so that
the rows of every sampling step are larger than the 126 MB L2:

  c2       verbo_cuda_sample, 256 x 151936 greedy + penalty over 128 ids
           (window_kernel, split_kernel greedy, merge_slices_kernel)
  c3       verbo_cuda_sample, 256 x 151936 top_k 50 + penalty over 256 ids
           (window_kernel, split_kernel top-k, merge_slices_kernel)
  c4       verbo_cuda_sample, 512 x 151936 full-vocabulary nucleus
           (nuc_a/b/c kernels and the resolve, general_list_kernel)
  staged   verbo_cuda_sample, 256 x 151936 top_k 100000 with min_p 0.02
           (general_kernel, 8-CTA clusters: top_k above 256)
  c5       verbo_cuda_shard_topk over 8 column shards + verbo_cuda_merge_sample,
           512 x 151936 (window_kernel, split_kernel emit, merge_slices_kernel,
           merge_kernel)
  batch    verbo_cuda_batch_accept + verbo_cuda_batch_step, 256 streams with
           C3 options (ring_accept_kernel, split_kernel, merge_slices_kernel)
  server   verbo_cuda_server_step, 4 requests over two option sets
           (state_gather_kernel and the sampling kernels)
  tail     verbo_cuda_tail_logits, 151936 x 896 Q8 head at 1 and 256 rows,
           Q4 at 8 rows, F32 at 1 row (tail_norm_kernel, tail_head_q_kernel,
           tail_head_f32_kernel); the tcgen05 head at 256 rows
           (VERBO_CUDA_TAIL_TCGEN05=1, tail_head_tc_kernel)

Between steps a one-element torch fill marks the boundary in a launch list,
and every input is made before the first step, so the only other kernels in
a capture are those markers (and the fill that creates the marker).  Each
step prints its name.
"""
from __future__ import annotations

import os

import numpy as np


def main() -> None:
    import torch

    import verbo_b200 as vb
    from verbo_b200 import workloads as wl

    vb.load_library()
    assert torch.cuda.is_available(), "the kernel tour needs a CUDA device"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    marker = torch.zeros(1, device=dev)

    def rows_of(name, rows):
        w = wl.WORKLOADS[name].with_rows(rows)
        x = torch.from_numpy(wl.make_rows_np(w)).to(dev)
        h, off = wl.make_hist_np(w)
        dh = None if h is None else torch.from_numpy(h).to(dev)
        do = None if off is None else torch.from_numpy(off).to(dev)
        st = np.array(vb.seed_states(w.sampler_seeds(0, rows)), dtype=np.uint64)
        rng = torch.from_numpy(st.view(np.int64).copy()).to(dev)
        return w, x, dh, do, rng

    # every input first
    c2 = rows_of("c2", 256)
    c3 = rows_of("c3", 256)
    c4 = rows_of("c4", 512)
    st = rows_of("c4", 256)
    c5 = rows_of("c5", 512)
    ob = vb.Sampling(**c3[0].sampling_kwargs())
    batch = vb.Batch(ob, 256)
    bh = c3[2].view(256, -1).cpu().numpy()
    srv = vb.Server(8, c2[0].vocab, max_window=256)
    sx = c2[1][:8].contiguous()
    tw = wl.TAIL
    heads = {}
    for dt in ("q8", "q4", "f32"):
        q, s, norm = tw.with_dtype(dt).make_head()
        heads[dt] = vb.Tail(dt, q, s, norm, tw.eps)
    hid = torch.from_numpy(tw.make_hidden_np(256)).to(dev)
    ncols = c5[0].vocab // 8
    cv = torch.empty(8, 512, 64, dtype=torch.float32, device=dev)
    ci = torch.empty(8, 512, 64, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()

    def step(name, fn):
        marker.fill_(1.0)
        fn()
        torch.cuda.synchronize()
        vb.check()
        print(name, flush=True)

    def sample(args, **over):
        w, x, dh, do, rng = args
        kw = w.sampling_kwargs()
        kw.update(over)
        vb.sample(x, vb.Sampling(**kw), rng=rng, hist=dh, hist_off=do)

    step("c2", lambda: sample(c2))
    step("c3", lambda: sample(c3))
    step("c4", lambda: sample(c4))
    step("staged", lambda: sample(st, temp=1.0, top_k=100000, top_p=0.95, min_p=0.02))

    def shards():
        w, x, dh, do, rng = c5
        o = vb.Sampling(**w.sampling_kwargs())
        for s in range(8):
            vb.shard_topk(x[:, s * ncols:(s + 1) * ncols], s * ncols, w.vocab, o, 64, dh, do,
                          cand_val=cv[s], cand_id=ci[s])
        vb.merge_sample(cv, ci, w.vocab, o, rng=rng)

    step("c5", shards)

    def batched():
        seeds = c3[0].sampler_seeds(0, 256)
        for i in range(256):
            batch.reset(i, int(seeds[i]))
            batch.accept(i, bh[i])
        batch.step(c3[1])

    step("batch", batched)

    def served():
        p = np.arange(4, dtype=np.int32)
        for i in range(4):
            o = vb.Sampling(temp=0.8, top_k=50, top_p=0.95, repeat=1.1, seed=100 + i) if i % 2 else \
                vb.Sampling(temp=0.0, repeat=1.2, seed=200 + i)
            srv.submit(p + i, o, 4)
        srv.prepare()
        srv.step(sx)

    step("server", served)
    step("tail q8 x1", lambda: heads["q8"].logits(hid[:1]))
    step("tail q8 x256", lambda: heads["q8"].logits(hid))
    step("tail q4 x8", lambda: heads["q4"].logits(hid[:8]))
    step("tail f32 x1", lambda: heads["f32"].logits(hid[:1]))
    os.environ["VERBO_CUDA_TAIL_TCGEN05"] = "1"
    step("tail q8 x256 tcgen05", lambda: heads["q8"].logits(hid))
    del os.environ["VERBO_CUDA_TAIL_TCGEN05"]
    for t in heads.values():
        t.close()
    batch.close()
    srv.close()
    print("kernel tour ok", flush=True)


if __name__ == "__main__":
    main()
