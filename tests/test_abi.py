"""CPU-only checks of the C-ABI boundary: the library loads, exports every
symbol include/*.h declares, and its metadata entry points answer like the
reference's QuantFormat / QGemvShape.  No kernel is launched here."""
import ctypes
import subprocess

import pytest

import objeta_b200
from objeta_b200 import QGemvShape, QuantFormat, _lib
from tests._util import ROOT, header_functions


def test_library_builds_in_tree():
    assert (ROOT / "objeta_b200" / "libobjeta_b200.so").exists()


def test_every_declared_symbol_is_exported():
    names = header_functions()
    assert len(names) >= 15
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "objeta_b200" / "libobjeta_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_library_is_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", str(ROOT / "objeta_b200" / "libobjeta_b200.so")],
                         capture_output=True, text=True).stdout
    archs = {tok for tok in out.split() if tok.startswith("sm_")}
    elf = [l for l in out.splitlines() if ".cubin" in l or "sm_" in l]
    assert elf, "no device code found"
    assert all("sm_100a" in l for l in elf), elf


def test_abi_version():
    assert _lib.load().objb_abi_version() == 100


@pytest.mark.parametrize("fmt,bb,label,kernel,scale", [
    (QuantFormat.Q4_0, 18, "q4_0", "q4_gemv", "F16"),
    (QuantFormat.Q5_0, 22, "q5_0", "q5_gemv", "F16"),
    (QuantFormat.IQ3_0, 14, "iq3_0", "iq3_gemv", "F16"),
    (QuantFormat.DeepSeekFp4E2M1, 17, "deepseek_fp4_e2m1", "fp4_e2m1_gemv", "F8_E8M0"),
])
def test_format_metadata(fmt, bb, label, kernel, scale):
    # quant.rs:33-96
    info = fmt._info()
    assert info.block_size == 32 == fmt.block_size()
    assert info.block_bytes == bb == fmt.block_bytes()
    assert info.format_label.decode() == label == fmt.format_label()
    assert info.kernel_name.decode() == kernel == fmt.kernel_name()
    assert info.scale_dtype.decode() == scale == fmt.scale_dtype()
    assert info.nibble_order.decode() == "low_first" == fmt.nibble_order()
    assert info.packed_values_per_byte == 2


def test_qgemv_shape_bytes():
    # BASELINE byte counts: Q4 4096x4096 -> 9,437,184; 151936x2048 -> 175,030,272
    assert QGemvShape.q4_0(4096, 4096).quantized_matrix_bytes() == 9_437_184
    assert QGemvShape.q4_0(151936, 2048).quantized_matrix_bytes() == 175_030_272
    assert QGemvShape.q5_0(151936, 2048).quantized_matrix_bytes() == 213_925_888
    assert QGemvShape.iq3_0(151936, 2048).quantized_matrix_bytes() == 136_134_656
    c = _lib.QGemvShapeC()
    _lib.call("objb_qgemv_shape_new", 0, 14336, 4096, ctypes.byref(c))
    assert c.quantized_matrix_bytes == 33_030_144 == QGemvShape.q4_0(14336, 4096).quantized_matrix_bytes()


def test_shape_rejects_non_multiple_cols():
    # quant.rs:1664-1670: message contains "multiple of block_size"
    c = _lib.QGemvShapeC()
    with pytest.raises(objeta_b200.CudaError) as ei:
        _lib.call("objb_qgemv_shape_new", 0, 4, 33, ctypes.byref(c))
    assert ei.value.kind == "InvalidInput"
    assert "multiple of block_size" in ei.value.source_message


def test_compute_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; this checks the no-GPU failure mode")
    with pytest.raises(objeta_b200.CudaError) as ei:
        objeta_b200.QuantBackend(0)
    assert ei.value.kind in ("Runtime", "Unsupported")


def test_compare_outputs_matches_reference_definition():
    """quant.rs:676-723 through the C ABI (host code, no GPU): against the
    oracle restatement, a mismatch error, and the empty / zero-norm cases."""
    import numpy as np
    from objeta_b200._lib import CudaError
    from objeta_b200.quant import compare_outputs
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    r = rng.standard_normal(1000).astype(np.float32)
    a = (r + rng.standard_normal(1000).astype(np.float32) * 1e-3).astype(np.float32)
    got = compare_outputs(r, a)
    ref = O.compare_outputs(r, a)
    assert abs(got.cosine_similarity - ref["cosine_similarity"]) <= 1e-6
    assert abs(got.relative_l2_error - ref["relative_l2_error"]) <= 1e-6 * max(1.0, ref["relative_l2_error"])
    assert got.max_abs_error == np.float32(ref["max_abs_error"])
    z = compare_outputs(np.zeros(4, np.float32), np.zeros(4, np.float32))
    assert (z.cosine_similarity, z.relative_l2_error, z.max_abs_error) == (1.0, 0.0, 0.0)
    try:
        compare_outputs(r, a[:-1])
        raise AssertionError("length mismatch accepted")
    except CudaError as e:
        assert e.kind == "InvalidInput" and "reference len 1000 != actual len 999" in e.source_message


def test_integration_binding_covers_the_header():
    """INTEGRATION.md's Rust extern block declares every function of
    include/*.h, so a maintainer can bind the whole ABI from it."""
    text = (ROOT / "INTEGRATION.md").read_text()
    block = text[text.index("## Rust FFI block"):text.index("## Status")]
    missing = [n for n in header_functions() if f"pub fn {n}(" not in block]
    assert not missing, f"not in the Rust block: {missing}"
