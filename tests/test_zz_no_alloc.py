"""persona_bgmv_fused_noalloc, called through the C ABI.

Some callers of this library cannot allocate device memory per call: an
inference engine that has already divided all of HBM into its own pools, or
a host binding without a device allocator.  For them the fused op has an
entry point that takes no workspace and allocates nothing; its scratch is a
fixed array inside the library.  These tests check that entry point against
the oracle and against the workspace entry point (persona_bgmv_fused), on
calls in a row that all use the shared array (more rows than the
decode-sized kernel takes, one of them at the row limit), plus a
decode-sized call, the row limit and the empty batch.

The file is collected last on purpose: it must pass both in a fresh process
and after every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

import capi_lib
from oracle import bgmv_oracle as O

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)  # the reference's tests/test_bgmv_cuda.py:29,43
MAX_ROWS = 8192  # PERSONA_NOALLOC_MAX_ROWS
SMALL_MAX_ROWS = 64  # PERSONA_SMALL_MAX_ROWS: above it the split kernel uses the array
NOALLOC_ROWS_STATUS = 8  # PERSONA_ERR_NOALLOC_ROWS


def _dev():
    return torch.device("cuda", 0)


def _t16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(_dev()).view(torch.bfloat16)


def _case(seed, T, K, N, R, S):
    rng = np.random.default_rng(seed)
    slots = rng.integers(-1, S, size=T).astype(np.int32)
    x = O.from_f32(rng.standard_normal((T, K)).astype(np.float32), "bf16")
    a = O.from_f32(rng.uniform(-1, 1, (S, R, K)).astype(np.float32) / np.sqrt(K), "bf16")
    b = O.from_f32((rng.standard_normal((S, N, R)) * 0.04).astype(np.float32), "bf16")
    y = O.from_f32(rng.standard_normal((T, N)).astype(np.float32), "bf16")
    return slots, x, a, b, y


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("K,N,R", [(1024, 512, 16)])
def test_noalloc_matches_oracle_on_calls_in_a_row(K, N, R):
    lib = capi_lib.load()
    S = 9
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    # three calls in a row on the shared array with different batches (its
    # plan, counters and partial sums sit at offsets that depend on T), the
    # last at the row limit; then a decode-sized call, which leaves it alone
    for call, T in enumerate((200, 1000, MAX_ROWS, 57)):
        assert (T > SMALL_MAX_ROWS) == (call < 3)
        slots, x, a, b, y0 = _case(100 + call, T, K, N, R, S)
        xd, ad, bd, sd = _t16(x), _t16(a), _t16(b), torch.from_numpy(slots).to(_dev())
        y_na = _t16(y0)
        capi_lib.check(lib.persona_bgmv_fused_noalloc(
            xd.data_ptr(), K, ad.data_ptr(), R * K, K, bd.data_ptr(), N * R, sd.data_ptr(), y_na.data_ptr(), N,
            T, K, N, R, S, capi_lib.BF16, err.data_ptr(), _stream()))
        # the same call through the workspace entry point
        y_ws = _t16(y0)
        ws_bytes = lib.persona_bgmv_workspace_size(T)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=_dev())
        capi_lib.check(lib.persona_bgmv_fused(
            xd.data_ptr(), K, ad.data_ptr(), R * K, K, bd.data_ptr(), N * R, sd.data_ptr(), y_ws.data_ptr(), N,
            T, K, N, R, S, capi_lib.BF16, ws.data_ptr(), ws_bytes, 0, err.data_ptr(), _stream()))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        y_ref = y0.copy()
        O.bgmv_forward_ref(x, a, b, slots, "bf16", y=y_ref)
        got = O.to_f32(_bits(y_na), "bf16")
        np.testing.assert_allclose(got, O.to_f32(y_ref, "bf16"), err_msg=f"T={T} vs oracle", **TOL)
        np.testing.assert_allclose(got, O.to_f32(_bits(y_ws), "bf16"), err_msg=f"T={T} vs workspace entry", **TOL)
        # rows without an adapter are left exactly as they were
        assert np.array_equal(_bits(y_na)[slots < 0], y0[slots < 0])


def test_noalloc_row_limit_and_empty_batch():
    lib = capi_lib.load()
    fake = 1 << 20  # never dereferenced: the call returns before any work
    st = lib.persona_bgmv_fused_noalloc(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64,
                                        MAX_ROWS + 1, 64, 64, 16, 4, capi_lib.BF16, None, _stream())
    assert st == NOALLOC_ROWS_STATUS
    assert b"PERSONA_NOALLOC_MAX_ROWS" in lib.persona_status_string(st)
    assert lib.persona_bgmv_fused_noalloc(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64,
                                          0, 64, 64, 16, 4, capi_lib.BF16, None, _stream()) == 0
