"""CPU-only checks of the native boundary: the CUDA library loads, exports
every entry point that include/bitnet_cuda.h declares, and the seeded input
generator is deterministic and follows the reference's quantisers."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "bitnet_cuda.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bitnet_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from bitnetrs_b200 import _native as N

    lib = N.cuda_lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.CUDA_LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(bitnet_cuda_\w+)", out))
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for f in declared_functions():
        assert hasattr(lib, f)


def test_python_bindings_cover_header():
    from bitnetrs_b200 import _native as N

    assert sorted(N.exported_cuda_symbols()) == declared_functions()


def test_build_recipe_targets_sm100a_only():
    """Every object is compiled for sm_100a alone (no PTX, no other SASS);
    the GPU test test_gpu_ops.py::test_kernels_loaded_for_sm100 checks the
    binary version the driver actually loads."""
    from bitnetrs_b200 import build

    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert build.NVCC_FLAGS[: len(build.ARCH)] == build.ARCH
    assert not any("compute_" in f and f not in build.ARCH for f in build.NVCC_FLAGS)


def test_invalid_shape_fields_without_gpu():
    """BitNetError::InvalidShape keeps `expected` and `got` apart across the C
    ABI; any other error clears them."""
    from bitnetrs_b200 import InvalidShape
    from bitnetrs_b200 import _native as N

    lib = N.cuda_lib()
    with pytest.raises(InvalidShape) as ei:
        N.check(lib.bitnet_cuda_model_check(None))
    assert ei.value.expected == "non-null model" and ei.value.got == "null"
    assert str(ei.value) == "invalid tensor shape: expected non-null model, got null"
    assert lib.bitnet_cuda_last_error_expected() == b"non-null model"
    h = C.c_void_p()
    if lib.bitnet_cuda_create(10**6, C.byref(h)) != 0:  # no such device: a backend error
        assert lib.bitnet_cuda_last_error_expected() == b"" and lib.bitnet_cuda_last_error_got() == b""


def test_version_and_error_without_gpu():
    from bitnetrs_b200 import _native as N

    lib = N.cuda_lib()
    assert b"sm_100a" in lib.bitnet_cuda_version()
    h = C.c_void_p()
    rc = lib.bitnet_cuda_create(0, C.byref(h))
    # no GPU in this container: BackendError, never a crash or a CPU fallback
    import torch

    if not torch.cuda.is_available():
        assert rc == 3
        assert lib.bitnet_cuda_last_error()


def test_synth_deterministic_and_thread_independent():
    from bitnetrs_b200 import synth

    synth.set_threads(1)
    a, sa = synth.ternary_absmean(7, 1001, 64, 200, 0.02)
    synth.set_threads(8)
    b, sb = synth.ternary_absmean(7, 1001, 64, 200, 0.02)
    synth.set_threads(0)
    assert sa == sb
    np.testing.assert_array_equal(a, b)
    c, _ = synth.ternary_absmean(8, 1001, 64, 200, 0.02)
    assert not np.array_equal(a, c)


def test_synth_absmean_matches_oracle():
    import oracle_lib as O
    from bitnetrs_b200 import synth

    rows, cols = 48, 100
    w = synth.normal_f32(11, 1003, rows * cols, 0.02)
    q = np.zeros(w.size, dtype=np.int8)
    s = C.c_float()
    assert O.lib().orc_absmean_quantize(O.p(w), w.size, O.p(q), C.byref(s)) == 0
    packed = np.zeros(rows * ((cols + 3) // 4), dtype=np.uint8)
    for r in range(rows):
        O.lib().orc_pack_ternary(O.p(q[r * cols:(r + 1) * cols].copy()), cols,
                                 packed[r * ((cols + 3) // 4):].ctypes.data)
    got, sg = synth.ternary_absmean(11, 1003, rows, cols, 0.02)
    assert sg == s.value
    np.testing.assert_array_equal(got, packed)
    # P(0) for N(0,s) weights under absmean: P(|z| < 0.5*sqrt(pi/2)) ~ 0.31
    zeros = np.mean(q == 0)
    assert 0.25 < zeros < 0.38


def test_synth_lm_head_matches_oracle_quantiser():
    import oracle_lib as O
    from bitnetrs_b200 import synth

    emb = synth.bf16_normal(3, 1, 37 * 64, 0.02)
    q, s = synth.quantize_bf16_rows_to_i8(emb, 37, 64)
    q2 = np.zeros_like(q)
    s2 = np.zeros_like(s)
    O.lib().orc_quantize_bf16_rows_to_i8(O.p(emb), 37, 64, O.p(q2), O.p(s2))
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)


def test_synth_ternary_codes_distribution():
    from bitnetrs_b200 import synth

    pk = synth.ternary_codes(5, 9, 256, 1024)
    codes = np.stack([(pk >> (2 * j)) & 3 for j in range(4)], -1).ravel()
    assert not np.any(codes == 3)
    frac = np.bincount(codes, minlength=3) / codes.size
    assert abs(frac[0] - 0.34) < 0.01 and abs(frac[1] - 0.32) < 0.01 and abs(frac[2] - 0.34) < 0.01


def test_kv_normal_moments():
    from bitnetrs_b200 import ModelConfig, synth

    cfg = ModelConfig(32, 64, 2, 4, 2, 96, 128, 10000.0, 1e-5)
    k, v = synth.kv_normal(1, 0, cfg, 100)
    assert k.shape == (2, 100, 32)
    assert abs(k.mean()) < 0.05 and abs(k.std() - 1.0) < 0.05
    assert not np.array_equal(k, v)


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++17")])
def test_header_compiles_as_plain_c_and_cpp(lang, std):
    # the boundary is consumed through FFIs (Rust bindgen/extern "C", ctypes),
    # so the header must stand alone as C99 as well as C++
    cc = "gcc" if lang == "c" else "g++"
    r = subprocess.run([cc, std, "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", lang, str(HEADER)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
