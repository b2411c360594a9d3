"""jq_csr / jq_csr_noalloc against a numpy restatement of the CSR contract.

The CSR is a pure function of the legal counts and ids (move_gen.py:1262-1307
defines the per-env order; here the ids are arbitrary): offsets are the
exclusive prefix sum of min(count, cap) with offsets[N] the total, and the
values are each env's first min(count, cap) ids, env after env.  Sizes cross
the kernels' block boundaries (1,024 envs per block sum, 8 envs per copy
block) and include counts of zero and above cap.
"""
import ctypes

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N

pytestmark = pytest.mark.gpu


def _csr_numpy(counts: np.ndarray, ids: np.ndarray, cap: int):
    c = np.minimum(counts, cap)
    off = np.zeros(len(counts) + 1, dtype=np.int64)
    off[1:] = np.cumsum(c)
    vals = np.concatenate([ids[e, : c[e]] for e in range(len(counts))]) if len(counts) else np.zeros(0)
    return off.astype(np.int32), vals.astype(np.int32)


@pytest.mark.parametrize("n,cap", [(1, 1), (7, 5), (8, 5), (9, 200), (1023, 64), (1024, 64), (1025, 64),
                                   (3000, 200), (70000, 48)])
def test_csr_matches_numpy(n, cap):
    N.build()
    L = N.lib()
    rng = np.random.default_rng(n * 1000 + cap)
    counts = rng.integers(0, cap + 3, n).astype(np.int32)  # some above cap: clamped
    counts[rng.random(n) < 0.1] = 0
    ids = rng.integers(0, 83521, (n, cap)).astype(np.int32)
    ref_off, ref_val = _csr_numpy(counts, ids, cap)
    dev = torch.device("cuda", 0)
    d_counts = torch.from_numpy(counts).to(dev)
    d_ids = torch.from_numpy(ids).to(dev)
    stream = torch.cuda.current_stream().cuda_stream
    scratch = torch.empty(max(int(L.jq_csr_scratch_ints(n)), 1), dtype=torch.int32, device=dev)
    for name in ("jq_csr", "jq_csr_noalloc"):
        off = torch.full((n + 1,), -7, dtype=torch.int32, device=dev)
        val = torch.full((max(int(ref_off[-1]), 1) + 16,), -7, dtype=torch.int32, device=dev)
        if name == "jq_csr":
            st = L.jq_csr(n, d_counts.data_ptr(), d_ids.data_ptr(), cap, off.data_ptr(), val.data_ptr(),
                          scratch.data_ptr(), ctypes.c_void_p(stream))
        else:
            st = L.jq_csr_noalloc(n, d_counts.data_ptr(), d_ids.data_ptr(), cap, off.data_ptr(), val.data_ptr(),
                                  ctypes.c_void_p(stream))
        N.check(st, name)
        torch.cuda.synchronize()
        got_off = off.cpu().numpy()
        got_val = val.cpu().numpy()
        np.testing.assert_array_equal(got_off, ref_off, err_msg=name)
        np.testing.assert_array_equal(got_val[: ref_off[-1]], ref_val, err_msg=name)
        assert (got_val[ref_off[-1]:] == -7).all(), f"{name} wrote past the last value"
