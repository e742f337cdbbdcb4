"""persona_bgmv_fused_noalloc: the fused op with its plan in the library's
fixed device array, called through the C ABI, against persona_bgmv_fused
with a caller workspace.  Two calls in a row with different batches; also
the row limit and the empty batch.  Collected last on purpose: it must pass
both in a fresh process and after every other test."""

import ctypes

import numpy as np
import pytest
import torch

import capi_lib
from oracle import bgmv_oracle as O

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-2, atol=1e-2)
MAX_ROWS = 8192  # PERSONA_NOALLOC_MAX_ROWS
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


@pytest.mark.parametrize("K,N,R", [(1024, 512, 16)])
def test_noalloc_matches_workspace_entry_point_twice(K, N, R):
    lib = capi_lib.load()
    S = 9
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    for call, T in enumerate((200, 57)):  # two calls in a row, different batches
        slots, x, a, b, y0 = _case(100 + call, T, K, N, R, S)
        xd, ad, bd, sd = _t16(x), _t16(a), _t16(b), torch.from_numpy(slots).to(_dev())
        y_ws = _t16(y0)
        ws_bytes = lib.persona_bgmv_workspace_size(T)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=_dev())
        capi_lib.check(lib.persona_bgmv_fused(
            xd.data_ptr(), K, ad.data_ptr(), R * K, K, bd.data_ptr(), N * R, sd.data_ptr(), y_ws.data_ptr(), N,
            T, K, N, R, S, capi_lib.BF16, ws.data_ptr(), ws_bytes, 0, err.data_ptr(), _stream()))
        y_na = _t16(y0)
        capi_lib.check(lib.persona_bgmv_fused_noalloc(
            xd.data_ptr(), K, ad.data_ptr(), R * K, K, bd.data_ptr(), N * R, sd.data_ptr(), y_na.data_ptr(), N,
            T, K, N, R, S, capi_lib.BF16, err.data_ptr(), _stream()))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = y_na.float().cpu().numpy()
        want = y_ws.float().cpu().numpy()
        np.testing.assert_allclose(got, want, **TOL)
        # rows without an adapter are left as they were
        assert np.array_equal(y_na.view(torch.int16).cpu().numpy()[slots < 0].view(np.uint16), y0[slots < 0])


def test_noalloc_row_limit_and_empty_batch():
    lib = capi_lib.load()
    fake = 1 << 20  # never dereferenced: the call returns before any work
    st = lib.persona_bgmv_fused_noalloc(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64,
                                        MAX_ROWS + 1, 64, 64, 16, 4, capi_lib.BF16, None, _stream())
    assert st == NOALLOC_ROWS_STATUS
    assert b"PERSONA_NOALLOC_MAX_ROWS" in lib.persona_status_string(st)
    assert lib.persona_bgmv_fused_noalloc(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64,
                                          0, 64, 64, 16, 4, capi_lib.BF16, None, _stream()) == 0
