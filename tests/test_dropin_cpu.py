"""The drop-in surface without a GPU: the torch.library registrations (operator names,
output shapes from their fake implementations, in-place arguments) and the raw-launch
stand-ins' ``kernel[grid](...)`` syntax."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode


def test_custom_ops_registered_with_shapes():
    from estudiocanciones_b200 import ops  # noqa: F401  (registers the operators)
    O = torch.ops.heartmula_b200
    with FakeTensorMode():
        x = torch.empty(8, 3072, dtype=torch.float16, device="cuda")
        w = torch.empty(5120, 3072, dtype=torch.int8, device="cuda")
        s = torch.empty(5120, dtype=torch.float16, device="cuda")
        assert O.int8_mm(x, w, s).shape == (8, 5120)
        assert O.int8_mm(x.reshape(2, 4, 3072), w, s).shape == (2, 4, 5120)
        assert O.rms(x, torch.empty(3072, dtype=torch.float16, device="cuda")).shape == (8, 3072)
        assert O.silu_mul(torch.empty(8, 16384, dtype=torch.float16, device="cuda")).shape == (8, 8192)
        a = torch.empty(4096, 3072, dtype=torch.float16, device="cuda")
        w13 = torch.empty(16384, 3072, dtype=torch.int8, device="cuda")
        s13 = torch.empty(16384, dtype=torch.float16, device="cuda")
        assert O.gemm_i8w(a, w13, s13, None, True).shape == (4096, 8192)
        assert O.gemm_i8w(a, w13, s13).shape == (4096, 16384)
    # in-place arguments are declared, so functionalisation knows what the kernels write
    schema = str(O.rope_cache.default._schema)
    assert "Tensor(a3!) q_out" in schema and "Tensor(a4!) kc" in schema and "Tensor(a5!) vc" in schema
    assert "Tensor(a4!) o" in str(O.attn.default._schema)


def test_raw_launch_names_take_the_grid_syntax():
    from estudiocanciones_b200 import kernels as K
    for name in ("_rope_cache", "_attn", "_attn_combine", "_silu_mul"):
        obj = getattr(K, name)
        with pytest.raises(TypeError):
            obj(1, 2, 3)                      # a bare call is not the reference's launch form
        assert callable(obj[(8, 4, 16)])      # obj[grid] -> a launcher
    # _attn_combine has nothing left to do once _attn merged its splits
    assert K._attn_combine[(1,)](None, None, None, None, HD=128, HDP=128, NSPLIT=16) is None
