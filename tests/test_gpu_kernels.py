"""Per-kernel parity on the GPU through the C ABI (gdc_linear, gdc_residual_layer_norm,
gdc_disentangled_attention) against the CPU oracle. Device memory comes from torch
(plumbing only); every kernel call goes through libgdc.so."""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import reference_forward as rf

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def _dev(a: np.ndarray):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


_KEEP: list = []


def _ptr(a: np.ndarray) -> int:
    """Device copy of `a` kept alive for the rest of the test session's current test."""
    t = _dev(a)
    _KEEP.append(t)
    return t.data_ptr()


@pytest.fixture(autouse=True)
def _release_kept():
    yield
    _torch().cuda.synchronize()
    _KEEP.clear()


def _host(t) -> np.ndarray:
    return t.cpu().numpy()


def _lib():
    from gliner_decide_metal_b200._lib import lib
    return lib


def _check(st):
    lib = _lib()
    assert st == 0, lib.gdc_last_error().decode()


@pytest.mark.parametrize("M,N,K,act", [
    (128, 256, 64, 0), (1, 128, 64, 0), (5, 2048, 1024, 2), (300, 384, 1024, 1), (1000, 3072, 1024, 0),
    (777, 1024, 4096, 0), (8192, 4096, 1024, 1), (8192, 1024, 4096, 0), (129, 256, 128, 2), (300, 256, 192, 0),
    (4096, 3072, 1088, 0)])
def test_linear_matches_numpy(M, N, K, act):
    """tcgen05 GEMM: out = act(a . w^T + b) vs float64 numpy on the same fp16 inputs."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(M * 7 + N + K + act))
    a = (rng.standard_normal((M, K), dtype=np.float32) * 0.5).astype(np.float16)
    w = (rng.standard_normal((N, K), dtype=np.float32) / math.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float16)
    da, dw, db = _dev(a), _dev(w), _dev(b)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_linear(da.data_ptr(), dw.data_ptr(), db.data_ptr(), out.data_ptr(), M, N, K, N, act, None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b.astype(np.float64)
    if act == 1:
        from scipy.special import erf
        ref = 0.5 * ref * (1 + erf(ref / math.sqrt(2)))
    elif act == 2:
        ref = np.maximum(ref, 0)
    got = _host(out).astype(np.float64)
    assert np.isfinite(got).all()
    # fp16 output rounding (2^-11 relative) plus fp32 accumulation
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("M,N,K,act", [
    (1, 4096, 1024, 1), (5, 3072, 1024, 0), (32, 3072, 1024, 0), (32, 1024, 1024, 0), (32, 1024, 4096, 0),
    (32, 4096, 1024, 1), (96, 1024, 4096, 0), (128, 2048, 1024, 2), (7, 1024, 192, 0)])
def test_linear_small_m_matches_numpy(M, N, K, act):
    """M <= 128 (a batch of one short row; BASELINE config 0's projections have M = 32): the
    skinny kernel, one narrow column tile per CTA over all of K, against float64 numpy; two
    calls in a row give the same bits."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(M * 13 + N + K + act))
    a = (rng.standard_normal((M, K), dtype=np.float32) * 0.5).astype(np.float16)
    w = (rng.standard_normal((N, K), dtype=np.float32) / math.sqrt(K)).astype(np.float16)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float16)
    da, dw, db = _dev(a), _dev(w), _dev(b)
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b.astype(np.float64)
    if act == 1:
        from scipy.special import erf
        ref = 0.5 * ref * (1 + erf(ref / math.sqrt(2)))
    elif act == 2:
        ref = np.maximum(ref, 0)
    outs = []
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        _check(_lib().gdc_linear(da.data_ptr(), dw.data_ptr(), db.data_ptr(), out.data_ptr(), M, N, K, N, act, None))
        torch.cuda.synchronize()
        _check(_lib().gdc_kernels_check_errors())
        got = _host(out)
        assert np.isfinite(got.astype(np.float32)).all()
        np.testing.assert_allclose(got.astype(np.float64), ref, rtol=2e-3, atol=2e-3)
        outs.append(got)
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))  # deterministic reduction


@pytest.mark.parametrize("M", [4096, 64])
def test_gelu_epilogue_is_correctly_rounded_nearly_everywhere(M):
    """The GELU of the FFN up-projection epilogue (MLXNN.gelu, DeBERTa.swift:421) on every fp16
    value step of [-12, 12]: an identity weight makes the accumulator the input exactly, so the
    output is fp16(GELU(x)) as the kernel evaluates it. Against float64 GELU rounded to fp16:
    at most 0.05% of outputs differ, each by one unit in the last place. M = 4096 runs on CTA
    pairs, M = 64 on the skinny kernel."""
    torch = _torch()
    from scipy.special import erf
    K = N = 1024
    x = np.linspace(-12.0, 12.0, M * K).astype(np.float16)
    a = x.reshape(M, K)
    w = np.eye(N, K, dtype=np.float16)
    b = np.zeros(N, dtype=np.float16)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_linear(_ptr(a), _ptr(w), _ptr(b), out.data_ptr(), M, N, K, N, 1, None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    got = _host(out).reshape(-1)
    xd = x.astype(np.float64)
    ref = (0.5 * xd * (1.0 + erf(xd / math.sqrt(2.0)))).astype(np.float16)
    differ = got.view(np.uint16) != ref.view(np.uint16)
    assert differ.mean() <= 5e-4, differ.mean()
    ulps = np.abs(got.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    same_sign = np.signbit(got) == np.signbit(ref)
    assert (ulps[differ & same_sign] <= 1).all()
    # a sign difference is only allowed between zero and the smallest subnormal
    assert (np.abs(got[differ & ~same_sign].astype(np.float32)) <= 6e-8).all()


def test_linear_leading_dimension():
    """Output written with ldo > N (the QKV projection writes into a wider buffer)."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(5))
    M, N, K, ldo = 200, 256, 128, 512
    a = (rng.standard_normal((M, K), dtype=np.float32) * 0.5).astype(np.float16)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.1).astype(np.float16)
    b = np.zeros(N, np.float16)
    out = torch.zeros((M, ldo), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_linear(_ptr(a), _ptr(w), _ptr(b), out.data_ptr(), M, N, K,
                             ldo, 0, None))
    torch.cuda.synchronize()
    got = _host(out)
    np.testing.assert_allclose(got[:, :N], a.astype(np.float32) @ w.astype(np.float32).T, rtol=2e-3, atol=2e-3)
    assert (got[:, N:] == 0).all()


@pytest.mark.parametrize("rows,cols,with_res", [(1, 1024, True), (37, 1024, True), (8192, 1024, True),
                                                 (64, 256, False), (3, 4096, True), (1500, 512, True),
                                                 (4099, 768, False), (2048, 256, True)])
def test_residual_layer_norm(rows, cols, with_res):
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(rows + cols))
    x = rng.standard_normal((rows, cols), dtype=np.float32).astype(np.float16)
    r = rng.standard_normal((rows, cols), dtype=np.float32).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(cols, dtype=np.float32)).astype(np.float16)
    bta = (0.1 * rng.standard_normal(cols, dtype=np.float32)).astype(np.float16)
    out = torch.empty((rows, cols), dtype=torch.float16, device="cuda")
    dr = _dev(r) if with_res else None
    _check(_lib().gdc_residual_layer_norm(_ptr(x), dr.data_ptr() if with_res else None,
                                          _ptr(g), _ptr(bta), out.data_ptr(), rows, cols,
                                          1e-7, None))
    torch.cuda.synchronize()
    s = (x + r).astype(np.float32) if with_res else x.astype(np.float32)  # fp16 add, as the reference
    ref = rf.layer_norm(s, g, bta, 1e-7)
    np.testing.assert_allclose(_host(out).astype(np.float32), ref, rtol=2e-3, atol=4e-3)


def test_residual_layer_norm_reference_recipe():
    """The reference's --kernel-test input (main.swift:194-225): x[i] = i/1024, residual 0,
    gamma 1, beta 0, [1, 1024], eps 1e-7."""
    torch = _torch()
    x = (np.arange(1024, dtype=np.float32) / 1024).astype(np.float16)[None]
    z = np.zeros_like(x)
    g = np.ones(1024, np.float16)
    b = np.zeros(1024, np.float16)
    out = torch.empty((1, 1024), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_residual_layer_norm(_ptr(x), _ptr(z), _ptr(g),
                                          _ptr(b), out.data_ptr(), 1, 1024, 1e-7, None))
    torch.cuda.synchronize()
    ref = rf.layer_norm(x.astype(np.float32), g, b, 1e-7)
    assert np.abs(_host(out).astype(np.float32) - ref).max() < 2e-3


def _attention_case(B, L, seed, lengths=None, scale=1.0):
    rng = np.random.Generator(np.random.PCG64(seed))
    H, d, E = 16, 64, 1024
    qkv = (rng.standard_normal((B * L, 3 * E), dtype=np.float32) * scale).astype(np.float16)
    rel = rng.standard_normal((512, E), dtype=np.float32)
    wq = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    wk = rng.standard_normal((E, E), dtype=np.float32) * 0.02
    pos = np.concatenate([rel @ wq.T, rel @ wk.T], axis=1).astype(np.float16)  # [512, 2E] PQ | PK
    if lengths is None:
        lengths = rng.integers(max(1, L // 4), L + 1, B)
    mask = np.zeros((B, L), np.float16)
    for b, n in enumerate(lengths):
        mask[b, :n] = 1
    return qkv, pos, mask


def _oracle_attention(qkv, pos, mask, B, L):
    H, d, E = 16, 64, 1024
    x = qkv.astype(np.float32).reshape(B, L, 3, H, d)
    q = x[:, :, 0].transpose(0, 2, 1, 3)
    k = x[:, :, 1].transpose(0, 2, 1, 3)
    v = x[:, :, 2].transpose(0, 2, 1, 3)
    pq = pos[:, :E].astype(np.float32).reshape(512, H, d).transpose(1, 0, 2)
    pk = pos[:, E:].astype(np.float32).reshape(512, H, d).transpose(1, 0, 2)
    c2p, p2c = rf.relative_indices(L)
    return rf.disentangled_attention(q, k, v, pq, pk, mask.astype(np.float32) > 0, c2p, p2c, fp16_rounding=True)


@pytest.mark.parametrize("B,L", [(1, 8), (2, 40), (3, 96), (1, 128), (2, 256), (1, 300), (1, 512), (2, 129)])
def test_attention_matches_oracle(B, L):
    torch = _torch()
    qkv, pos, mask = _attention_case(B, L, seed=B * 1000 + L)
    ctx = torch.full((B * L, 1024), float("nan"), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_disentangled_attention(_ptr(qkv), _ptr(pos), _ptr(mask),
                                             ctx.data_ptr(), B, L, 16, None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    got = _host(ctx).astype(np.float32).reshape(B, L, 1024)
    ref = _oracle_attention(qkv, pos, mask, B, L)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=4e-3)


def test_attention_reference_relative_recipe():
    """Deterministic inputs in the style of the reference's --relative-kernel-test
    (main.swift:141-192): q[i]=(i%13)/13, k[i]=(7i%17)/17, v from (5i%23)/23, relative
    tables (3i%19)/19 and (5i%23)/23; keys 6 and 7 of 8 masked."""
    torch = _torch()
    B, L, E = 1, 8, 1024
    n = B * L * 3 * E
    i = np.arange(n)
    qkv = np.empty((B * L, 3 * E), np.float32)
    qkv[:, :E] = ((i[: B * L * E] % 13) / 13).reshape(B * L, E)
    qkv[:, E:2 * E] = (((i[: B * L * E] * 7) % 17) / 17).reshape(B * L, E)
    qkv[:, 2 * E:] = (((i[: B * L * E] * 5) % 23) / 23).reshape(B * L, E)
    j = np.arange(512 * E)
    pos = np.concatenate([(((j * 5) % 23) / 23).reshape(512, E), (((j * 3) % 19) / 19).reshape(512, E)], axis=1)
    qkv, pos = qkv.astype(np.float16), pos.astype(np.float16)
    mask = np.array([[1, 1, 1, 1, 1, 1, 0, 0]], np.float16)
    ctx = torch.empty((B * L, E), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_disentangled_attention(_ptr(qkv), _ptr(pos), _ptr(mask),
                                             ctx.data_ptr(), B, L, 16, None))
    torch.cuda.synchronize()
    ref = _oracle_attention(qkv, pos, mask, B, L)
    np.testing.assert_allclose(_host(ctx).astype(np.float32).reshape(ref.shape), ref, rtol=1e-2, atol=4e-3)


def test_attention_masked_keys_get_zero_weight():
    """Changing V (and K) at masked key positions must not change any output."""
    torch = _torch()
    B, L = 2, 64
    qkv, pos, mask = _attention_case(B, L, seed=9, lengths=[40, 17])
    qkv2 = qkv.copy().reshape(B, L, 3 * 1024)
    qkv2[0, 40:, 1024:] = 7.0
    qkv2[1, 17:, 1024:] = -3.0
    outs = []
    for q in (qkv, qkv2.reshape(B * L, -1)):
        ctx = torch.empty((B * L, 1024), dtype=torch.float16, device="cuda")
        _check(_lib().gdc_disentangled_attention(_ptr(q), _ptr(pos), _ptr(mask),
                                                 ctx.data_ptr(), B, L, 16, None))
        outs.append(_host(ctx))
    torch.cuda.synchronize()
    assert np.array_equal(outs[0], outs[1])


def test_attention_config1_draw_matches_oracle():
    """BASELINE config 1 exactly: B=32, H=16, L=256, q/k/v N(0,1), PQ / PK = rel N(0,1)
    projected by N(0, 0.02) weights, key lengths U[64, 256]. The kernel runs the whole batch;
    8 batch rows (all 16 heads, every query position) are compared with the oracle. Rows
    are independent, so comparing a slice of the batch is exact."""
    torch = _torch()
    B, L = 32, 256
    rng = np.random.Generator(np.random.PCG64(20261))
    lengths = rng.integers(64, L + 1, B)
    qkv, pos, mask = _attention_case(B, L, seed=20262, lengths=lengths)
    ctx = torch.full((B * L, 1024), float("nan"), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_disentangled_attention(_ptr(qkv), _ptr(pos), _ptr(mask), ctx.data_ptr(), B, L, 16, None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    got = _host(ctx).astype(np.float32).reshape(B, L, 1024)
    assert np.isfinite(got).all()
    rows = [0, 3, 7, 12, 18, 21, 26, 31]
    sub = np.concatenate([qkv.reshape(B, L, -1)[b] for b in rows]).reshape(len(rows) * L, -1)
    ref = _oracle_attention(sub, pos, mask[rows], len(rows), L)
    np.testing.assert_allclose(got[rows], ref, rtol=1e-2, atol=4e-3)


@pytest.mark.parametrize("B,L", [(1, 8), (2, 40), (2, 129), (1, 300), (1, 512)])
def test_attention_scalar_kernel_matches_oracle(B, L):
    """The CUDA-core cross-check kernel (used below at sizes the oracle cannot reach) is
    itself pinned to the oracle at small shapes."""
    torch = _torch()
    qkv, pos, mask = _attention_case(B, L, seed=B * 3000 + L)
    ctx = torch.full((B * L, 1024), float("nan"), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_disentangled_attention_scalar(_ptr(qkv), _ptr(pos), _ptr(mask), ctx.data_ptr(), B, L, 16,
                                                    None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    got = _host(ctx).astype(np.float32).reshape(B, L, 1024)
    ref = _oracle_attention(qkv, pos, mask, B, L)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=4e-3)


@pytest.mark.parametrize("B,L", [(32, 256), (4, 512), (8, 64), (3, 200)])
def test_attention_tensor_core_matches_scalar_kernel(B, L):
    """Full BASELINE config-1 shape (B=32, H=16, L=256, key lengths U[64, 256]) and L=512:
    the tcgen05 kernel against the CUDA-core kernel on the device (the CPU oracle is too
    slow at this size)."""
    torch = _torch()
    rng = np.random.Generator(np.random.PCG64(L + B))
    lengths = rng.integers(min(64, L), L + 1, B)
    qkv, pos, mask = _attention_case(B, L, seed=77 + L, lengths=lengths)
    pq, pp, pm = _ptr(qkv), _ptr(pos), _ptr(mask)
    a = torch.empty((B * L, 1024), dtype=torch.float16, device="cuda")
    b = torch.empty((B * L, 1024), dtype=torch.float16, device="cuda")
    _check(_lib().gdc_disentangled_attention(pq, pp, pm, a.data_ptr(), B, L, 16, None))
    _check(_lib().gdc_disentangled_attention_scalar(pq, pp, pm, b.data_ptr(), B, L, 16, None))
    torch.cuda.synchronize()
    _check(_lib().gdc_kernels_check_errors())
    x, y = _host(a).astype(np.float32), _host(b).astype(np.float32)
    assert np.isfinite(x).all()
    np.testing.assert_allclose(x, y, rtol=1e-2, atol=4e-3)


def test_device_wait_timeout_is_reported_and_device_stays_usable():
    """Failure detection without a fault: a kernel's bounded wait on a barrier that nothing
    completes gives up after 2 ms, sets the timeout bit, returns; the host sees
    GDC_ERR_TIMEOUT once, and the next kernel call works."""
    torch = _torch()
    lib = _lib()
    assert lib.gdc_kernels_check_errors() == 0
    _check(lib.gdc_selftest_wait_timeout(2000, None))
    torch.cuda.synchronize()
    assert lib.gdc_kernels_check_errors() == 9  # GDC_ERR_TIMEOUT
    assert b"time limit" in lib.gdc_last_error()
    assert lib.gdc_kernels_check_errors() == 0  # cleared
    assert lib.gdc_selftest_wait_timeout(0, None) == 3  # GDC_ERR_INVALID_INPUT
    rng = np.random.Generator(np.random.PCG64(3))
    a = rng.standard_normal((256, 64), dtype=np.float32).astype(np.float16)
    w = rng.standard_normal((256, 64), dtype=np.float32).astype(np.float16)
    b = np.zeros(256, np.float16)
    out = torch.empty((256, 256), dtype=torch.float16, device="cuda")
    _check(lib.gdc_linear(_ptr(a), _ptr(w), _ptr(b), out.data_ptr(), 256, 256, 64, 256, 0, None))
    torch.cuda.synchronize()
    _check(lib.gdc_kernels_check_errors())
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    np.testing.assert_allclose(_host(out).astype(np.float64), ref, rtol=2e-3, atol=2e-3)
