"""The allocation-free CSR entry point agrees with the allocating one.

jq_csr_noalloc exists for callers that cannot allocate device memory (a
process whose CUDA allocator already owns the HBM budget, or a thin FFI host
holding only the buffers it was given): it keeps its scratch in a fixed
device array inside libjq.so.  This test calls it through the C ABI twice in
a row, on two different legal-move sets, and checks offsets and values
against jq_csr, which takes caller-provided scratch.  It also checks the
size limit.  The file is named so pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from junqi_b200 import _native as N
from junqi_b200 import tables
from junqi_b200.env import JunqiEnvB200

pytestmark = pytest.mark.gpu


def test_csr_noalloc_matches_allocating_entry_point_on_consecutive_calls():
    L = N.lib()
    env = JunqiEnvB200(3000, pool=tables.build_setup_pool(32, seed=8), with_obs=False, with_mask=False)
    env.reset(seed=21)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        env.ply(env.sample_uniform(21, call + 1), seed=21, ply=call + 1)
        ref_off, ref_val = env.csr()
        off = torch.full_like(ref_off, -7)
        val = torch.full_like(ref_val, -7)
        N.check(L.jq_csr_noalloc(env.n, env.counts.data_ptr(), env.ids.data_ptr(), env.cap, off.data_ptr(),
                                 val.data_ptr(), stream), "jq_csr_noalloc")
        torch.cuda.synchronize()
        total = int(ref_off[-1])
        assert total > 0
        assert torch.equal(off, ref_off), f"offsets differ on call {call}"
        assert torch.equal(val[:total], ref_val[:total]), f"values differ on call {call}"
        counts = env.counts.cpu().numpy()
        assert np.array_equal(np.diff(off.cpu().numpy()), counts)


def test_csr_noalloc_rejects_sizes_beyond_its_scratch():
    L = N.lib()
    x = torch.zeros(4, dtype=torch.int32, device="cuda")
    st = L.jq_csr_noalloc((1 << 20) + 1, x.data_ptr(), x.data_ptr(), 1, x.data_ptr(), x.data_ptr(), None)
    assert st == 4
    assert b"JQ_NOALLOC_MAX_ENVS" in L.jq_last_error()
