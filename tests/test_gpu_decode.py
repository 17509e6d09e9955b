"""verbo_cuda_batch_decode on the reference's decode loops.

tests/golden/decode_models.npz holds, per case, B >= 2 concurrent generations
on the reference's tiny checkpoints, each an independent verbo::generate run
(src/sampler.cpp:111-181), with every pick's id and the hidden row its logits
came from.  The B generations step together through the C ABI: one call per
step takes the B hidden rows (host memory on even steps, device memory on odd
ones), runs the logits tail on the device into rows the batch owns and picks +
accepts for every generation; the ids must equal the reference's picks (the
oracle's margin rule applies only to rows on a decision boundary, and no
fixture row is one).  The logits never reach the host.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import pyoracle as po
from tests.decode_fixture import load_cases
from tests.gpu_util import compare

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_batch_decode_matches_reference_generations(cuda_lib, case):
    import verbo_b200 as vb

    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    tail = vb.Tail(case.head_dtype, case.q, case.s, case.norm, case.eps)
    batch = vb.Batch(vb.Sampling(**case.opts), case.B)
    for b in range(case.B):
        batch.reset(b, int(case.seeds[b]))
        batch.accept(b, case.prompts[b])
    # the oracle on the same rows, for the boundary rule
    o = po.sampling(**case.opts)
    states = po.seed_states(case.seeds)
    hist = [list(p) for p in case.prompts]
    stats = torch.zeros(case.B * vb.ROW_STATS_BYTES, dtype=torch.uint8, device="cuda")
    for j in range(case.steps):
        rows = np.ascontiguousarray(case.x[:, j])
        if j % 2 == 0:
            got = batch.decode(tail, rows)                       # host rows in, host ids out
        else:
            got = batch.decode(tail, torch.from_numpy(rows).cuda(), stats=stats).cpu().numpy()
        act = [b for b in range(case.B) if j < case.npicks[b]]
        logits, _, _ = po.logits_tail(case.head_dtype, case.q, case.s, case.norm, case.eps, case.x[act, j])
        h = np.concatenate([np.array(hist[b], dtype=np.int32) for b in act])
        off = np.cumsum([0] + [len(hist[b]) for b in act]).astype(np.int64)
        st = np.ascontiguousarray(states[act])
        ora, ost = po.sample_rows(logits, o, st, h, off)
        states[act] = st
        assert ora.tolist() == case.ids[act, j].tolist()
        n = compare(got[act], case.ids[act, j], ost, f"{case.name} step {j}")
        assert n == 0, f"{case.name} step {j}: {n} boundary rows differ"
        # every generation accepts its own pick, as the batch did on the device
        for b in range(case.B):
            if b in act:
                hist[b].append(int(got[b]))
    vb.check()
    tail.close()
    batch.close()


def test_batch_decode_rejects_bad_arguments(cuda_lib):
    import verbo_b200 as vb

    case = CASES[0]
    dim = case.x.shape[2]
    tail = vb.Tail(case.head_dtype, case.q, case.s, case.norm, case.eps)
    batch = vb.Batch(vb.Sampling(**case.opts), case.B)
    lib = vb.load_library()
    with pytest.raises(vb.VerboCudaError):
        batch.decode(tail, np.zeros((case.B + 1, dim), dtype=np.float32))   # one row per generation
    assert lib.verbo_cuda_batch_decode(batch._h, tail._h, None, dim, None, None, None) == -1
    assert b"NULL" in lib.verbo_cuda_last_error()
    h = torch.zeros(case.B, dim, dtype=torch.float32, device="cuda")
    out = torch.zeros(case.B, dtype=torch.int32, device="cuda")
    assert lib.verbo_cuda_batch_decode(batch._h, tail._h, h.data_ptr(), dim - 1, out.data_ptr(), None, None) == -1
    assert b"ldx" in lib.verbo_cuda_last_error()
    tail.close()
    batch.close()
