"""gdc_disentangled_attention_noalloc (the allocation-free attention entry point) against
gdc_disentangled_attention on the same inputs, through the C ABI, on two calls in a row.

The file name makes pytest collect it last. Device buffers come from torch (plumbing); the
entry point itself keeps its scratch in a static device array."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, E = 16, 1024


def _case(B: int, L: int, seed: int):
    rng = np.random.Generator(np.random.PCG64(seed))
    qkv = rng.standard_normal((B * L, 3 * E), dtype=np.float32).astype(np.float16)
    rel = rng.standard_normal((512, E), dtype=np.float32)
    wq = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    wk = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    pos = np.concatenate([rel @ wq.T, rel @ wk.T], axis=1).astype(np.float16)
    lengths = rng.integers(max(1, L // 4), L + 1, B)
    mask = np.zeros((B, L), np.float16)
    for b, n in enumerate(lengths):
        mask[b, :n] = 1
    return qkv, pos, mask


def test_noalloc_attention_matches_allocating_entry_point_twice():
    import torch
    from gliner_decide_metal_b200._lib import lib

    def check(st):
        assert st == 0, lib.gdc_last_error().decode()

    for i, (B, L, seed) in enumerate([(4, 200, 11), (2, 512, 12)]):
        qkv, pos, mask = _case(B, L, seed)
        dq, dp, dm = (torch.from_numpy(x).cuda() for x in (qkv, pos, mask))
        ref = torch.full((B * L, E), float("nan"), dtype=torch.float16, device="cuda")
        got = torch.full((B * L, E), float("nan"), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        check(lib.gdc_disentangled_attention(dq.data_ptr(), dp.data_ptr(), dm.data_ptr(), ref.data_ptr(),
                                             B, L, H, None))
        torch.cuda.synchronize()
        check(lib.gdc_kernels_check_errors())
        free_before = torch.cuda.mem_get_info()[0]
        check(lib.gdc_disentangled_attention_noalloc(dq.data_ptr(), dp.data_ptr(), dm.data_ptr(), got.data_ptr(),
                                                     B, L, H, None))
        torch.cuda.synchronize()
        if i == 0:
            # the call allocates nothing: device memory the driver reports free did not shrink
            # (the static array was mapped with the library's module, before the first call)
            assert torch.cuda.mem_get_info()[0] >= free_before
        # same kernel, same relative table, same static work split: the fp16 bits agree exactly
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
        assert np.isfinite(got.cpu().numpy().astype(np.float32)).all()


def test_noalloc_attention_rejects_sizes_beyond_its_scratch():
    import torch
    from gliner_decide_metal_b200._lib import lib

    x = torch.zeros(16, dtype=torch.float16, device="cuda")
    p = x.data_ptr()
    st = lib.gdc_disentangled_attention_noalloc(p, p, p, p, 1, 513, H, None)
    assert st == 10  # GDC_ERR_UNSUPPORTED
    assert b"512" in lib.gdc_last_error()
