"""The C-ABI library builds, loads and exports exactly what include/hexgen2_b200.h declares;
the product path refuses to run without CUDA (no CPU fallback)."""
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "hexgen2_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hx_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    from hexgen2_b200 import _lib
    lib = _lib.lib()
    assert lib.hx_abi_version() == 1
    declared = declared_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == declared


def test_library_symbols_are_in_the_dynamic_table():
    import subprocess
    from hexgen2_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T (hx_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_workspace_queries_need_no_gpu():
    from hexgen2_b200 import _lib
    lib = _lib.lib()
    assert lib.hx_gemm_workspace(1, 64, 64, 0, _lib.HX_F32) == 0
    # Decode-shaped bf16 GEMMs reduce inside a cluster: no workspace.
    assert lib.hx_gemm_workspace(32, 4096, 4096, 0, _lib.HX_BF16) == 0
    assert lib.hx_gemm_workspace(300, 512, 2048, 0, _lib.HX_BF16) > 0
    # Prefill shapes with enough 256 x 256 items run on CTA pairs (no workspace); small ones
    # on single-SM tiles; m <= 64 is decode-shaped.
    assert lib.hx_gemm_kernel_kind(900, 4096, 4096, _lib.HX_BF16) == 2
    assert lib.hx_gemm_workspace(900, 4096, 4096, 0, _lib.HX_BF16) == 0
    assert lib.hx_gemm_kernel_kind(300, 512, 2048, _lib.HX_BF16) == 1
    assert lib.hx_gemm_kernel_kind(128, 22016, 4096, _lib.HX_BF16) == 1
    assert lib.hx_gemm_kernel_kind(32, 4096, 4096, _lib.HX_BF16) == 3
    assert lib.hx_gemm_kernel_kind(900, 4096, 4096, _lib.HX_F32) == 0
    # head_dim 32: one key split, no partials; head_dim 128: the balanced path's partials.
    assert lib.hx_decode_attention_workspace(1, 32, 32, 16) == 0
    assert lib.hx_decode_attention_workspace(1, 32, 128, 16) > 0
    assert lib.hx_decode_attention_workspace(1, 32, 128, 8192) > 0


def test_ops_refuse_cpu_tensors():
    from hexgen2_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm(torch.zeros(2, 8), torch.zeros(4, 8))
    with pytest.raises(ValueError, match="CUDA"):
        ops.rmsnorm(torch.zeros(2, 8), torch.ones(8), 1e-6)
    q, cache = torch.zeros(3, 2, 8), torch.zeros(1, 4, 2, 1, 8)
    with pytest.raises(ValueError, match="CUDA"):
        ops.prefill_attention_varlen(q, cache, [3], [0], 1, 0.5, torch.empty_like(q))
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm_qkv_rotary_varlen(torch.zeros(3, 16), torch.zeros(32, 16), [3], [0], 2, 1, 8,
                                   torch.zeros(4, 4), torch.zeros(4, 4), cache, q)


def test_native_engine_refuses_cpu(tmp_path):
    """The native engine has no CPU path (the explicitly chosen hf-reference engine is
    transformers' own model, tests/test_engine_hf_cpu.py)."""
    from hexgen2_b200 import Engine
    from hexgen2_b200.fixture import create
    folder = create(tmp_path / "m", seed=0)
    with pytest.raises(ValueError):
        Engine(folder, device="cpu", dtype="float32")
    with pytest.raises(ValueError):
        Engine(folder, engine="native", device="cpu", dtype="float32")


def test_graft_build_compiles_for_sm100a():
    from hexgen2_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert build.LIB.exists()
