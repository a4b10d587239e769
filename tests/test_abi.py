"""CPU tests of the C ABI: the library builds for sm_100a, loads, and exports
every entry point that include/remora_b200.h declares.  No compute calls."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(remora_b200_\w+)\s*\(", text))
    return sorted(names)


def test_library_builds_and_exports_every_declared_symbol():
    from remora_b200 import build

    path = build.build()
    lib = ctypes.CDLL(path)
    syms = declared_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_mirror_binds_every_declared_symbol():
    import remora_b200

    remora_b200.lib()
    assert set(declared_symbols()) <= set(remora_b200._SIGNATURES)


def test_recognise_and_errors_without_gpu():
    import remora_b200 as rb

    assert rb.recognise("elementwise") and rb.recognise("projection") and rb.recognise("gemm")
    assert not rb.recognise("softmax_v2")
    # argument validation happens before any CUDA call
    rc = rb.lib().remora_b200_gemm_bf16(None, None, None, 1, 8, 8, 8, 8, 8, 8, 0, 0, 0, 0, None)
    assert rc == rb.ERR_INVALID and "null" in rb.last_error()
    rc = rb.lib().remora_b200_relu_bias_f32(None, None, None, 1, 0, None)
    assert rc == rb.ERR_INVALID


def test_stream_keys_agree_with_oracle():
    import oracle
    import remora_b200 as rb

    for s in (1, 10, 34):
        for seed in (42, 7):
            assert rb.stream_key(s, seed) == oracle.stream_key(s, seed)
