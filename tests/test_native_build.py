"""CPU checks of the native build: the C-ABI library loads and exports every
function include/*.h declares, the torch ops register the reference's exact
schemas, and host-side argument validation returns status codes (no kernel
is launched: every call here fails validation before touching the GPU)."""

import ctypes

import pytest
import torch

import capi_lib


@pytest.fixture(scope="module")
def built():
    import importlib.util
    import sys
    from pathlib import Path

    spec = importlib.util.spec_from_file_location(
        "persona_build", Path(capi_lib.ROOT) / "multi-lora-llm-kernel_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    return True


def test_library_exports_header_symbols(built):
    lib = capi_lib.load()
    declared = capi_lib.declared_symbols()
    assert {"persona_bgmv_shrink", "persona_bgmv_expand", "persona_bgmv_fused"} <= declared
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(capi_lib.SIGNATURES) <= declared
    assert lib.persona_abi_version() == 1


def test_reference_schemas_registered(built):
    import persona._C  # noqa: F401

    s = {n: str(getattr(torch.ops.persona, n).default._schema)
         for n in ("bgmv_shrink", "bgmv_expand", "gemv_fp16")}
    # reference csrc/bindings.cpp:20-22, byte for byte
    assert s["bgmv_shrink"] == "persona::bgmv_shrink(Tensor x, Tensor a_pool, Tensor slots, Tensor(a!) v) -> ()"
    assert s["bgmv_expand"] == "persona::bgmv_expand(Tensor v, Tensor b_pool, Tensor slots, Tensor(a!) y) -> ()"
    assert s["gemv_fp16"] == "persona::gemv_fp16(Tensor x, Tensor W, Tensor(a!) y) -> ()"
    assert persona._C.noop() == 0


def test_workspace_size_matches_layout(built):
    lib = capi_lib.load()
    def a256(n):
        return (n + 255) // 256 * 256

    for T in (0, 1, 8, 512, 16384):
        tp = (T + 3) // 4 * 4
        plan = 32 + 4 * tp + 16 * tp                  # header, perm, items
        sync = a256(plan)                              # counters, per-item state of 8 problems
        vfinal = a256(sync + 4 * (16 + 2 * 8 * tp))    # v per problem and plan position, 64 floats

        def total(problems):
            parts = a256(vfinal + problems * tp * 64 * 4)  # 1024 partial-v slots of 16 x 64 floats
            return parts + 1024 * 16 * 64 * 4

        assert lib.persona_bgmv_workspace_size(T) == total(1)
        # + per-row slots, then the tensor-core kernel's partial-v pieces:
        # two of 128 x 32 fp32 for each of at most 160 CTAs
        assert lib.persona_sgmv_workspace_size(T) == a256(total(1) + 4 * tp) + 2 * 160 * 128 * 64 * 4
        for p in (1, 3, 8):
            assert lib.persona_bgmv_multi_workspace_size(T, p) == total(p)
        assert lib.persona_bgmv_multi_workspace_size(T, 9) == 0


def test_host_validation_codes(built):
    lib = capi_lib.load()
    fake = 1 << 20  # 16-byte aligned, never dereferenced: validation fails first
    wsp = fake
    big = lib.persona_bgmv_workspace_size(512)  # enough for every call below
    # unsupported dtype
    assert lib.persona_bgmv_fused(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64, 8, 64,
                                  64, 16, 4, 7, wsp, big, 0, None, None) == 3
    # rank 12 is not a fused/expand rank
    assert lib.persona_bgmv_fused(fake, 64, fake, 64 * 12, 64, fake, 64 * 12, fake, fake, 64, 8, 64,
                                  64, 12, 4, 0, wsp, big, 0, None, None) == 5
    # K not a multiple of 8
    assert lib.persona_bgmv_shrink(fake, 68, fake, 68 * 16, 68, fake, fake, 8, 68, 16, 4, 0,
                                   wsp, big, 0, None, None) == 2
    # misaligned x
    assert lib.persona_bgmv_shrink(fake + 8, 64, fake, 64 * 16, 64, fake, fake, 8, 64, 16, 4, 0,
                                   wsp, big, 0, None, None) == 4
    # workspace too small
    assert lib.persona_bgmv_expand(fake, fake, 64 * 16, fake, fake, 64, 512, 64, 16, 4, 0, wsp, 64,
                                   0, None, None) == 6
    # unknown flag
    assert lib.persona_bgmv_expand(fake, fake, 64 * 16, fake, fake, 64, 8, 64, 16, 4, 0, wsp, big,
                                   8, None, None) == 1
    # T == 0 is a no-op
    assert lib.persona_bgmv_fused(fake, 64, fake, 64 * 16, 64, fake, 64 * 16, fake, fake, 64, 0, 64,
                                  64, 16, 4, 0, wsp, big, 0, None, None) == 0
    assert b"R must be" in lib.persona_status_string(5)


def test_ops_refuse_cpu_tensors(built):
    from persona import ops

    assert ops.has_cuda_ops()
    x = torch.zeros(2, 64, dtype=torch.float16)
    a = torch.zeros(2, 16, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be CUDA"):
        ops.bgmv_shrink(x, a, torch.zeros(2, dtype=torch.int32))
