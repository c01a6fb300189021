"""Host-side behaviour of the dispatcher ops and the module that needs no GPU:
schemas match the reference, Meta kernels give the right shapes, argument errors mirror
the reference, and the module's packed checkpoint format is the reference's."""
import numpy as np
import pytest
import torch

import nanoquant_b200 as nq
from oracle import oracle as orc

from .golden_data import GOLDEN


def test_reference_schemas_registered():
    s = str(torch.ops.binary_kernels.nanoquant_dyn_forward.default._schema)
    assert s.startswith("binary_kernels::nanoquant_dyn_forward(Tensor x, Tensor scale_g, Tensor Ubits, "
                        "Tensor? scale_l, Tensor Vbits, Tensor scale_h, int num_thread_stage1=128")
    assert "num_acc_stage1=4" in s and "num_pipeline_stage2=2" in s
    s = str(torch.ops.binary_kernels.marlin_nanoquant_forward.default._schema)
    assert "Tensor(a!) workspace" in s and "Tensor weight_u, Tensor weight_v" in s
    assert hasattr(torch.ops.binary_kernels, "marlin_onebit_forward")


def test_meta_shapes():
    x = torch.empty(3, 4096, device="meta", dtype=torch.float16)
    s2 = torch.empty(4096, device="meta", dtype=torch.float16)
    vb = torch.empty(1126, 128, device="meta", dtype=torch.int32)
    ub = torch.empty(11008, 36, device="meta", dtype=torch.int32)
    s1 = torch.empty(11008, device="meta", dtype=torch.float16)
    y = torch.ops.binary_kernels.nanoquant_dyn_forward(x, s2, vb, None, ub, s1)
    assert y.shape == (3, 11008) and y.dtype == torch.float16
    assert torch.ops.nq_b200.linear(x, s2, vb, None, ub, s1).shape == (3, 11008)
    assert torch.ops.nq_b200.gemm(x, s2, vb, None, ub, s1, True).shape == (3, 11008)
    p = torch.ops.nq_b200.pack_signs(torch.empty(5, 33, device="meta", dtype=torch.int8), "half2", False)
    assert p.shape == (5, 2) and p.dtype == torch.int32


def test_marlin_meta_shapes_and_checks():
    """The Marlin ops' Meta kernels: output shapes and the reference's argument checks
    (gemm.cpp:37-56) without a GPU."""
    x = torch.empty(7, 512, device="meta", dtype=torch.float16)
    vb = torch.empty(32, 128, device="meta", dtype=torch.int32)   # in 512, padded rank 256
    ub = torch.empty(16, 64, device="meta", dtype=torch.int32)    # rank 256, out 128
    ws = torch.empty(64, device="meta", dtype=torch.int32)
    y = torch.ops.binary_kernels.marlin_nanoquant_forward(x, vb, ub, None, None, None, ws)
    assert y.shape == (7, 128) and y.dtype == torch.float16
    y1 = torch.ops.binary_kernels.marlin_onebit_forward(x, vb, None, None, ws)
    assert y1.shape == (7, 256)
    with pytest.raises(RuntimeError, match="k dimension mismatch"):
        torch.ops.binary_kernels.marlin_onebit_forward(x, ub, None, None, ws)
    p = torch.ops.nq_b200.pack_marlin(torch.empty(128, 64, device="meta", dtype=torch.int8), False)
    assert p.shape == (4, 64) and p.dtype == torch.int32


def test_marlin_packer_aliases_match_reference_names():
    from nanoquant_b200 import kernel_utils as ku
    assert ku.marlin_onebit_packer is ku.pack_binary_marlin
    assert ku.marlin_nanoquant_packer is ku.pack_binary_marlin_fused
    assert ku.MARLIN_MIN_MAX_PAR == 32


def test_get_kernel_function_resolves_reference_op():
    f = nq.get_kernel_function("nanoquant", torch.float16, "dynamic")
    assert f is torch.ops.binary_kernels.nanoquant_dyn_forward
    with pytest.raises(AttributeError):
        nq.get_kernel_function("nope", torch.float16, "dynamic")


def test_binary_kernels_module_alias():
    import binary_kernels  # noqa: F401  (what the reference imports)


def test_packer_error_behaviour_matches_reference():
    with pytest.raises(TypeError):
        nq.pack_binary_gemv(torch.ones(2, 2, dtype=torch.int32))
    with pytest.raises(ValueError):
        nq.pack_binary_gemv(torch.ones(2, 2, dtype=torch.int8), "msb_first")
    with pytest.raises(ValueError):
        nq.unpack_binary_gemv(torch.zeros(3, dtype=torch.int32), (3, 1))
    with pytest.raises(ValueError):
        nq.unpack_binary_gemv(torch.zeros(3, 1, dtype=torch.int32), (3, 40))
    with pytest.raises(RuntimeError):  # no host fallback
        nq.pack_binary_gemv(torch.ones(2, 2, dtype=torch.int8))


def test_module_state_dict_matches_reference_format():
    """Same keys and planes as the reference module's state_dict for the golden 7x5 r3 case."""
    m = nq.NanoQuantLinear(5, 7, 3, bias=True, packed=True)
    U = orc.random_signs(77, 7, 3)
    V = orc.random_signs(78, 3, 5)
    with torch.no_grad():
        m.U_packed.copy_(torch.from_numpy(orc.pack(U, "lsb_first")))
        m.V_packed.copy_(torch.from_numpy(orc.pack(V, "lsb_first")))
        m.scale_pre.fill_(1)
        m.scale_post.fill_(1)
    sd = m.state_dict()
    assert sorted(sd.keys()) == sorted(str(k) for k in GOLDEN["sd_keys"])
    for k in ("U_packed", "V_packed", "U_shape", "V_shape"):
        np.testing.assert_array_equal(sd[k].numpy(), GOLDEN[f"sd_{k}"])
    # round trip into a fresh module, strict, without dense expansion
    m2 = nq.NanoQuantLinear(5, 7, 3, bias=True, packed=True)
    m2.load_state_dict(sd, strict=True)
    np.testing.assert_array_equal(m2.U_packed.numpy(), GOLDEN["sd_U_packed"])
    assert m2.scale_mid is None and not hasattr(m2, "U")


def test_module_load_rejects_bad_planes():
    m = nq.NanoQuantLinear(5, 7, 3, packed=True)
    sd = m.state_dict()
    sd["U_packed"] = torch.zeros(7, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError):
        m.load_state_dict(sd, strict=True)


def test_module_requires_cuda_for_kernels():
    m = nq.NanoQuantLinear(64, 32, 16, packed=True)
    with pytest.raises(RuntimeError):
        m._prepare_kernel("gemv", torch.float16)
    with pytest.raises(NotImplementedError):
        m._prepare_kernel("gemlite", torch.float16)
