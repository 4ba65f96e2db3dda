"""The allocation-free split+merge attention entry point.

Some callers cannot give the library scratch memory (their memory pool owns
the whole device, or cudaMalloc's implicit synchronisation is off-limits on
their hot path).  gpt2b_attention_forward_kv_large_bf16_noalloc keeps the
split partials in a fixed array inside the library instead.  This test calls
it through the C ABI three times in a row and checks each result against the
regular entry point, which takes caller-allocated partial buffers; it also
checks that a size beyond the built-in array is refused.

Collected last on purpose (file name), so a run stopping at the first failure
has already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_attention_matches_regular_entry_point(cuda, gpt2b):
    lib = gpt2b.lib()
    NH, hs, maxT = 12, 64, 1024
    rng = np.random.default_rng(77)
    kv = torch.from_numpy(rng.standard_normal(2 * NH * maxT * hs, dtype=np.float32)).to("cuda", torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    # calls in a row with different sizes; the third has fewer splits than the second, so a
    # merge that read a stale slot left by the previous call would change the output
    for call, (pos, S) in enumerate([(700, 8), (1023, 13), (1023, 5)]):
        qkv = torch.from_numpy(rng.standard_normal(3 * NH * hs, dtype=np.float32)).to("cuda", torch.bfloat16)
        d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        # the regular entry point with caller-allocated partials
        po = torch.empty(NH * S * hs, device="cuda")
        pl, pm = torch.empty(NH * S, device="cuda"), torch.empty(NH * S, device="cuda")
        want = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
        gpt2b.check(lib.gpt2b_attention_forward_kv_large_bf16(_vp(want), _vp(qkv), _vp(kv), 1, NH, hs, maxT,
                                                              _vp(d_pos), stream, _vp(po), _vp(pl), _vp(pm), S))
        got = torch.full((NH * hs,), float("nan"), device="cuda", dtype=torch.bfloat16)
        gpt2b.check(lib.gpt2b_attention_forward_kv_large_bf16_noalloc(_vp(got), _vp(qkv), _vp(kv), 1, NH, hs, maxT,
                                                                      _vp(d_pos), S, stream))
        torch.cuda.synchronize()
        g, w = got.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.isfinite(g).all(), call
        assert rel_err(g, w) < 1e-2, call  # the BF16 attention tolerance used by the other tests
        # the same split and merge kernels on the same inputs: the outputs are bit-identical
        assert torch.equal(got, want), call


def test_noalloc_attention_refuses_sizes_beyond_its_array(cuda, gpt2b):
    lib = gpt2b.lib()
    NH, hs, maxT = 64, 64, 64
    kv = torch.zeros(2 * NH * maxT * hs, device="cuda", dtype=torch.bfloat16)
    qkv = torch.zeros(3 * NH * hs, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(NH * hs, device="cuda", dtype=torch.bfloat16)
    d_pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.gpt2b_attention_forward_kv_large_bf16_noalloc(_vp(out), _vp(qkv), _vp(kv), 1, NH, hs, maxT, _vp(d_pos),
                                                           33, None)  # 64 * 33 = 2112 > 2048 partial rows
    assert rc == gpt2b.ERR_INVALID_ARG
