"""NF4 base linears on the GPU against the oracle: the device quantiser and
dequantiser bit for bit, the decode GEMM within atol = rtol = 1e-2 at every
row count it packs differently (1 to 64 rows, and more in 64-row launches),
several weights per launch, split and unsplit K, strided y, determinism, and
the C ABI's argument checks."""

import ctypes

import numpy as np
import pytest
import torch

import capi_lib
from oracle import nf4_oracle as Q
from persona import nf4, ops

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)


def _dev():
    return torch.device("cuda", 0)


def _weights(seed, N, K, scale=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * scale).astype(np.float16)
    w[3, 64:128] = 0  # a zero block
    w[N - 1, K - 1] = np.float16(0.75)  # an outlier
    return w


@pytest.mark.parametrize("N,K", [(128, 128), (256, 384), (1024, 4096), (384, 1152)])
def test_device_quantiser_and_dequantiser_match_the_oracle_bit_for_bit(N, K):
    w = _weights(N * 7 + K, N, K)
    packed_ref, off_ref = Q.quantize(w.astype(np.float32))
    q = nf4.quantize(torch.from_numpy(w).to(_dev()))
    assert float(q.offset.item()) == float(off_ref)
    assert np.array_equal(q.packed.cpu().numpy(), packed_ref)
    deq = nf4.dequantize(q).cpu().numpy()
    assert np.array_equal(deq.view(np.uint16), Q.dequantize_f16(packed_ref, off_ref, N, K).view(np.uint16))


@pytest.mark.parametrize("M", [1, 3, 8, 13, 16, 31, 32, 64, 100])
def test_linear_matches_the_oracle(M):
    N, K = 512, 1024
    w = _weights(M, N, K)
    q = nf4.quantize(torch.from_numpy(w).to(_dev()))
    rng = np.random.default_rng(100 + M)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = nf4.linear(torch.from_numpy(x).to(_dev()), [q], dense_above=1 << 30)[0]
    ops.check_errors(_dev())
    want = Q.linear_ref(x, q.packed.cpu().numpy(), np.float32(q.offset.item()), N, K)
    np.testing.assert_allclose(y.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)


def test_several_weights_per_launch_split_and_unsplit_k():
    """q / k / v shapes sharing x (K 4096: split K), then a wide weight whose
    K of 256 is never split; each against the oracle and the dense path."""
    rng = np.random.default_rng(5)
    M = 8
    for shapes in ([(1024, 4096), (256, 4096), (256, 4096)], [(2048, 256), (128, 256)]):
        K = shapes[0][1]
        qs = [nf4.quantize(torch.from_numpy(_weights(i + K, N, K)).to(_dev())) for i, (N, _) in enumerate(shapes)]
        x = rng.standard_normal((M, K)).astype(np.float16)
        xd = torch.from_numpy(x).to(_dev())
        ys = nf4.linear(xd, qs)
        dense = nf4.linear(xd, qs, dense_above=0)
        ops.check_errors(_dev())
        for q, y, yd, (N, _) in zip(qs, ys, dense, shapes):
            want = Q.linear_ref(x, q.packed.cpu().numpy(), np.float32(q.offset.item()), N, K)
            np.testing.assert_allclose(y.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)
            np.testing.assert_allclose(yd.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)


def test_decode_shapes_strided_output_and_determinism():
    """The down projection (K 14336, many splits) into a column window of a
    wider y; two launches give the same bits."""
    N, K, M = 4096, 14336, 8
    g = torch.Generator(device=_dev()).manual_seed(9)
    w = (torch.randn(N, K, generator=g, device=_dev()) * 0.02).half()
    q = nf4.quantize(w)
    x = torch.randn(M, K, generator=g, device=_dev()).half()
    wide = torch.full((M, N + 64), 7.0, dtype=torch.float16, device=_dev())
    y = wide[:, 32:32 + N]
    nf4.linear(x, [q], outs=[y])
    first = y.clone()
    nf4.linear(x, [q], outs=[y])
    ops.check_errors(_dev())
    assert torch.equal(first, y)
    assert torch.all(wide[:, :32] == 7) and torch.all(wide[:, 32 + N:] == 7)
    ref = (x.float() @ nf4.dequantize(q).float().t())
    torch.testing.assert_close(y.float(), ref, **TOL)


def test_c_abi_checks_arguments():
    lib = capi_lib.load()
    N, K, M = 256, 256, 4
    q = nf4.quantize(torch.from_numpy(_weights(1, N, K)).to(_dev()))
    x = torch.randn(M, K, device=_dev()).half()
    y = torch.empty(M, N, device=_dev(), dtype=torch.float16)
    P = capi_lib.Nf4Problem
    prob = P(q.packed.data_ptr(), q.offset.data_ptr(), x.data_ptr(), K, y.data_ptr(), N, N, K)
    arr = (P * 1)(prob)
    ws_bytes = lib.persona_nf4_linear_workspace_size(arr, 1)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=_dev())
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi_lib.check(lib.persona_nf4_linear(arr, 1, M, ws.data_ptr(), ws_bytes, err.data_ptr(), st))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = Q.linear_ref(x.cpu().numpy(), q.packed.cpu().numpy(), np.float32(q.offset.item()), N, K)
    np.testing.assert_allclose(y.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)
    assert lib.persona_nf4_linear(arr, 1, M, ws.data_ptr(), ws_bytes - 1, err.data_ptr(), st) == 6
    assert lib.persona_nf4_linear(arr, 0, M, ws.data_ptr(), ws_bytes, err.data_ptr(), st) == 1
    bad = (P * 1)(P(q.packed.data_ptr(), q.offset.data_ptr(), x.data_ptr(), K, y.data_ptr(), N, N, 200))
    assert lib.persona_nf4_linear(bad, 1, M, ws.data_ptr(), ws_bytes, err.data_ptr(), st) == 2
    assert lib.persona_nf4_packed_bytes(N, K) == (N // 128) * (K // 128) * 8464
    assert lib.persona_nf4_packed_bytes(100, K) == 0


@pytest.mark.parametrize("M", [3, 8, 64])
def test_linear_with_addend_matches_the_oracle(M):
    """y = fp16(x W^T + addend): the addend joins before the one rounding,
    on the split-K path (K 4096) and the unsplit one (K 256)."""
    rng = np.random.default_rng(40 + M)
    for N, K in ((1024, 4096), (384, 256)):
        q = nf4.quantize(torch.from_numpy(_weights(M + K, N, K)).to(_dev()))
        x = rng.standard_normal((M, K)).astype(np.float16)
        add = rng.standard_normal((M, N)).astype(np.float32)
        y = nf4.linear(torch.from_numpy(x).to(_dev()), [q], addends=[torch.from_numpy(add).to(_dev())])[0]
        ops.check_errors(_dev())
        w = Q.dequantize_f32(q.packed.cpu().numpy(), np.float32(q.offset.item()), N, K).astype(np.float64)
        want = (x.astype(np.float64) @ w.T + add).astype(np.float16)
        np.testing.assert_allclose(y.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)


@pytest.mark.parametrize("M", [1, 8, 20])
def test_problems_of_different_k_in_one_launch(M):
    """Four linears with their own x and K in one launch through the C ABI
    (1018 chunks, three to four per CTA on a B200): the CTAs' equal chunk
    ranges cross problem boundaries where the chunks per tile change (3, 25,
    1, 13), tiles are cut into pieces of different lengths, and one tile is a
    single chunk.  Each y against the oracle; a second launch gives the same
    bits."""
    lib = capi_lib.load()
    shapes = [(384, 384), (4096, 3200), (128, 128), (2048, 1664)]
    rng = np.random.default_rng(70 + M)
    qs, xs, ys, probs = [], [], [], []
    for i, (N, K) in enumerate(shapes):
        q = nf4.quantize(torch.from_numpy(_weights(200 + i, N, K)).to(_dev()))
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16)).to(_dev())
        y = torch.full((M, N), 3.0, dtype=torch.float16, device=_dev())
        qs.append(q), xs.append(x), ys.append(y)
        probs.append(capi_lib.Nf4Problem(q.packed.data_ptr(), q.offset.data_ptr(), x.data_ptr(), K, y.data_ptr(), N,
                                         N, K))
    arr = (capi_lib.Nf4Problem * len(probs))(*probs)
    ws_bytes = lib.persona_nf4_linear_workspace_size(arr, len(probs))
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=_dev())
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi_lib.check(lib.persona_nf4_linear(arr, len(probs), M, ws.data_ptr(), ws_bytes, err.data_ptr(), st))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    first = [y.clone() for y in ys]
    for q, x, y, (N, K) in zip(qs, xs, ys, shapes):
        want = Q.linear_ref(x.cpu().numpy(), q.packed.cpu().numpy(), np.float32(q.offset.item()), N, K)
        np.testing.assert_allclose(y.cpu().numpy().astype(np.float32), want.astype(np.float32), **TOL)
    capi_lib.check(lib.persona_nf4_linear(arr, len(probs), M, ws.data_ptr(), ws_bytes, err.data_ptr(), st))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for a, b in zip(first, ys):
        assert torch.equal(a, b)


def test_bitsandbytes_checkpoint_through_the_kernels():
    """A weight in bitsandbytes' NF4 storage (double-quantised scales,
    restated in oracle/bnb_nf4.py), converted by nf4.from_bitsandbytes and
    applied by the decode GEMM and by the dequantiser: against the fp32
    product with the weight that storage describes (tolerance: this format's
    scale step, plus fp16 rounding)."""
    from oracle import bnb_nf4

    rng = np.random.default_rng(11)
    N, K, M = 512, 1024, 8
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    st = bnb_nf4.quantize_nf4(w)
    q = nf4.from_bitsandbytes(torch.from_numpy(st["packed"]).cuda(), torch.from_numpy(st["absmax"]).cuda(),
                              st["shape"], torch.from_numpy(st["quant_map"]), blocksize=64,
                              nested_absmax=torch.from_numpy(st["nested_absmax"]).cuda(),
                              nested_quant_map=torch.from_numpy(st["nested_quant_map"]).cuda(),
                              nested_offset=st["nested_offset"], nested_blocksize=256)
    w_bnb = bnb_nf4.dequantize(st)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = nf4.linear(torch.from_numpy(x).cuda(), [q])[0].float().cpu().numpy()
    want = x.astype(np.float64) @ w_bnb.astype(np.float64).T
    np.testing.assert_allclose(y, want, rtol=2e-2, atol=2e-2)
    wd = nf4.dequantize(q).float().cpu().numpy()
    np.testing.assert_allclose(wd, w_bnb, rtol=1e-2, atol=2e-4)
    ops.check_errors(torch.device("cuda", 0))
