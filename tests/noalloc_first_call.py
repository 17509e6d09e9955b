"""Worker of tests/test_zz_no_alloc.py: in a fresh process, the first call of
the library is verbo_cuda_sample_noalloc.  Prints one JSON line: the device
memory that first call took (CUDA's lazy module loading places the library's
module, with its fixed scratch array, on the device then), the memory later
calls took (none), and whether the ids equal verbo_cuda_sample's."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import verbo_b200 as vb  # noqa: E402
from oracle import pyoracle as po  # noqa: E402


def main():
    torch.cuda.set_device(0)
    rows, V = 64, 151936
    g = np.random.default_rng(7)
    x = torch.from_numpy((g.standard_normal((rows, V)) * 2).astype(np.float32)).cuda()
    states = po.seed_states(np.arange(1, rows + 1, dtype=np.uint64)).view(np.int64)
    rng_a = torch.from_numpy(states.copy()).cuda()
    rng_b = torch.from_numpy(states.copy()).cuda()
    got = torch.empty(rows, dtype=torch.int32, device="cuda")
    want = torch.empty(rows, dtype=torch.int32, device="cuda")
    o = vb.Sampling(temp=0.8, top_k=50, top_p=0.95)
    vb.load_library()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    vb.sample_noalloc(x, o, rng=rng_b, out=got)  # the library's first call
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        vb.sample_noalloc(x, o, rng=rng_b, out=got)
    torch.cuda.synchronize()
    free2 = torch.cuda.mem_get_info()[0]
    vb.check()
    # the allocating entry point, three calls from the same states
    for _ in range(3):
        vb.sample(x, o, rng=rng_a, out=want)
    vb.check()
    print(json.dumps({"first_call_bytes": free0 - free1, "later_calls_bytes": free1 - free2,
                      "ids_equal": bool(torch.equal(got, want) and torch.equal(rng_a, rng_b))}))


if __name__ == "__main__":
    main()
