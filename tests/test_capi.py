"""C ABI checks that need no GPU: the library loads, exports every symbol the header
declares, and rejects bad arguments on the host before touching a device."""
import ctypes
import os
import re

import pytest

from nanoquant_b200 import _lib

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADERS = [os.path.join(INCLUDE, h) for h in ("nq_b200.h", "nq_decoder.h")]


def declared_symbols():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"NQ_API\s+[\w\s\*]*?\b(nq_\w+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = declared_symbols()
    for n in ("nq_pack_signs", "nq_unpack_signs", "nq_repack_signs", "nq_gemv", "nq_gemv_workspace_bytes",
              "nq_gemm", "nq_gemm_workspace_bytes", "nq_workspace_reset", "nq_workspace_status",
              "nq_rmsnorm", "nq_rope_cache", "nq_decode_attention", "nq_decode_attention_rope", "nq_silu_mul"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.CUDA_LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) <= set(_lib._SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.cuda_lib()
    assert lib.nq_abi_version() == 1
    assert lib.nq_status_string(0) == b"ok"
    assert b"timed out" in lib.nq_status_string(_lib.NQ_ERR_DEVICE_TIMEOUT)


def test_workspace_sizes():
    lib = _lib.cuda_lib()
    # control block + 8 interm rows of round_up(rank, 64) floats
    assert lib.nq_gemv_workspace_bytes(1, 1126) == 256 + 8 * 1152 * 4
    assert lib.nq_gemv_workspace_bytes(64, 1126) == lib.nq_gemv_workspace_bytes(1, 1126)
    assert lib.nq_gemv_workspace_bytes(1, 0) == 0
    assert lib.nq_gemm_workspace_bytes(2048, 2054) >= 256
    # attention: control block + counters (256-byte rounded) + [batch][hq][chunks][130] floats;
    # 64-position chunks while a head has at most 64 of them, longer chunks beyond
    assert lib.nq_decode_attention_workspace_bytes(1, 32, 128, 2400) == 256 + 256 + 32 * 38 * 130 * 4
    assert lib.nq_decode_attention_workspace_bytes(2, 8, 128, 9000) == 256 + 256 + 2 * 8 * 47 * 130 * 4
    assert lib.nq_decode_attention_workspace_bytes(1, 32, 128, 0) == 0


@pytest.mark.parametrize("case", ["head_dim", "group", "small_ws", "unaligned_ws", "null_q"])
def test_attention_rejects_bad_arguments_on_host(case):
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: every check runs before a launch
    ws_bytes = lib.nq_decode_attention_workspace_bytes(1, 8, 128, 512)
    args = dict(q=fake, hq=8, hkv=2, d=128, ws=fake, wsb=ws_bytes)
    if case == "head_dim":
        args["d"] = 64
    elif case == "group":
        args["hq"], args["hkv"] = 9, 3  # group of 3 is not supported
    elif case == "small_ws":
        args["wsb"] = ws_bytes - 1
    elif case == "unaligned_ws":
        args["ws"] = ctypes.c_void_p(0x10010)
    elif case == "null_q":
        args["q"] = None
    for rope in (False, True):
        if rope:
            st = lib.nq_decode_attention_rope(0, args["q"], fake, fake, fake, fake, fake, fake, 1, args["hq"],
                                              args["hkv"], args["d"], 512, 10000.0, args["ws"], args["wsb"], None)
        else:
            st = lib.nq_decode_attention(0, args["q"], fake, fake, fake, fake, 1, args["hq"], args["hkv"], args["d"],
                                         512, args["ws"], args["wsb"], None)
        assert st != 0, (case, rope)
        assert lib.nq_last_error_message()


@pytest.mark.parametrize("case", ["null_x", "bad_dtype", "zero_batch", "small_ws"])
def test_gemv_rejects_bad_arguments_on_host(case):
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    args = dict(dtype=0, x=fake, batch=1, in_f=64, s2=fake, vb=fake, rank=16, smid=None, ub=fake, out_f=32,
                s1=fake, y=fake, ws=fake, wsb=lib.nq_gemv_workspace_bytes(1, 16))
    expect = {"null_x": _lib.NQ_ERR_INVALID_ARGUMENT, "bad_dtype": _lib.NQ_ERR_UNSUPPORTED,
              "zero_batch": _lib.NQ_ERR_INVALID_ARGUMENT, "small_ws": _lib.NQ_ERR_WORKSPACE}[case]
    if case == "null_x":
        args["x"] = None
    elif case == "bad_dtype":
        args["dtype"] = 7
    elif case == "zero_batch":
        args["batch"] = 0
    else:
        args["wsb"] = 16
    st = lib.nq_gemv(args["dtype"], args["x"], args["batch"], args["in_f"], args["s2"], args["vb"], args["rank"],
                     args["smid"], args["ub"], args["out_f"], args["s1"], args["y"], args["ws"], args["wsb"], None)
    assert st == expect
    assert lib.nq_last_error_message()


def test_pack_rejects_bad_arguments_on_host():
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)
    assert lib.nq_pack_signs(None, 2, 2, 0, fake, None, None) == _lib.NQ_ERR_INVALID_ARGUMENT
    assert lib.nq_pack_signs(fake, 0, 2, 0, fake, None, None) == _lib.NQ_ERR_INVALID_ARGUMENT
    assert lib.nq_pack_signs(fake, 2, 2, 5, fake, None, None) == _lib.NQ_ERR_INVALID_ARGUMENT
    assert lib.nq_unpack_signs(fake, 2, -1, 0, fake, None) == _lib.NQ_ERR_INVALID_ARGUMENT
    assert lib.nq_repack_signs(fake, 2, 2, 0, 9, fake, None) == _lib.NQ_ERR_INVALID_ARGUMENT
    with pytest.raises(_lib.NQError):
        _lib.check(_lib.NQ_ERR_INVALID_ARGUMENT)


@pytest.mark.parametrize("case", ["mode", "no_x2", "no_weight", "unaligned", "act", "batch"])
def test_group_ex_rejects_bad_input_descriptors_on_host(case):
    lib = _lib.cuda_lib()
    fake = 0x10000  # never dereferenced: the descriptor checks run first
    inp = _lib.GemvInput(x_mode=1, eps=1e-5, x=fake, x2=fake, norm_weight=fake, residual_out=fake)
    layer = _lib.GemvLayer(scale_pre=fake, v_bits=fake, rank=64, scale_mid=None, u_bits=fake, out_features=64,
                           scale_post=fake, y=fake)
    batch, act = 1, 0
    if case == "mode":
        inp.x_mode = 9
    elif case == "no_x2":
        inp.x_mode, inp.x2 = 3, None
    elif case == "no_weight":
        inp.norm_weight = None
    elif case == "unaligned":
        inp.x2 = fake + 2
    elif case == "act":
        act = 2  # bit beyond the single layer
    elif case == "batch":
        batch = 9
    st = lib.nq_gemv_group_ex(0, ctypes.byref(inp), batch, 256, 1, ctypes.byref(layer), act, None, 0, None)
    assert st in (_lib.NQ_ERR_INVALID_ARGUMENT, _lib.NQ_ERR_UNSUPPORTED), st
    assert lib.nq_last_error_message()
