"""Host-side logic of the drop-in layer (no GPU): backend selection semantics,
ingest validation, error reporting and the reference-compatible surface."""

import types

import pytest
import torch

from mirai_b200 import backend as bk
from mirai_b200 import experts as ex
from mirai_b200 import tables


def _fake_reference_int8(E=4, I=128, H=64, group=0):
    m = types.SimpleNamespace()
    m._quant_format = "int8"
    m.num_experts = E
    m.w1_int8 = torch.zeros(E, I, H, dtype=torch.int8)
    m.w3_int8 = torch.zeros(E, I, H, dtype=torch.int8)
    m.w2_int8 = torch.zeros(E, H, I, dtype=torch.int8)
    for k in ("w1", "w2", "w3"):
        setattr(m, f"{k}_scale", torch.ones(*getattr(m, f"{k}_int8").shape[:-1], 1))
        setattr(m, f"{k}_group_size", group)
    m.expert_rotation = lambda key: None
    m.expert_lora = {}
    return m


def test_backend_protocol_attributes():
    b = bk.B200MoEKernelBackend()
    assert b.name == "b200" and b.direct_only
    assert b.supports_routed_output_observer is False
    assert callable(b.execute_direct)


def test_backend_strict_fails_fast_and_auto_falls_back_on_cpu_tokens():
    m = _fake_reference_int8()
    tokens = torch.zeros(8, 64)
    scores = torch.ones(8, 2) / 2
    idx = torch.zeros(8, 2, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="moe_kernel_backend='b200'.*CUDA"):
        bk.B200MoEKernelBackend(strict=True).execute_direct(m, tokens, scores, idx)
    assert bk.B200MoEKernelBackend(strict=False).execute_direct(m, tokens, scores, idx) is None


def test_backend_module_checks():
    m = _fake_reference_int8()
    assert bk.B200MoEKernelBackend.module_reason(m) is None
    m.expert_lora = {"w2": object()}
    assert "LoRA" in bk.B200MoEKernelBackend.module_reason(m)
    m.expert_lora = {}
    m.has_logical_expert_aliases = lambda: True
    assert "aliases" in bk.B200MoEKernelBackend.module_reason(m)


def test_registry_hook():
    assert isinstance(bk.build_moe_kernel_backend("b200", direct_routed=True), bk.B200MoEKernelBackend)
    with pytest.raises(ValueError):
        bk.build_moe_kernel_backend("torch", direct_routed=True)
    with pytest.raises(ValueError):
        bk.build_moe_kernel_backend("b200", direct_routed=False)


def test_rotated_int8_binding_rules():
    """The fixed block-Hadamard format binds (on CUDA buffers); what the fused
    path cannot run is refused with the reason: a learned rotation matrix,
    a group that is not a power of 4, gate/up groups that differ."""
    from mirai_b200._lib import MiraiError
    m = _fake_reference_int8(group=16)
    m.expert_rotation = lambda key: torch.eye(16)
    with pytest.raises(MiraiError, match="learned rotation"):
        ex.GroupedExpertWeights.from_module(m)
    m = _fake_reference_int8(group=32)
    with pytest.raises(MiraiError, match="power of 4"):
        ex.GroupedExpertWeights.from_module(m)
    m = _fake_reference_int8(group=16)
    m.w3_group_size = 64
    with pytest.raises(MiraiError, match="gate/up rotation groups differ"):
        ex.GroupedExpertWeights.from_module(m)
    # plain and rotated layers both reach the descriptor step (which needs CUDA tensors)
    with pytest.raises(ValueError, match="CUDA"):
        ex.GroupedExpertWeights.from_module(_fake_reference_int8(group=16))


def test_best_group_size_follows_the_reference_rule():
    assert ex.best_group_size(3072) == 256 and ex.best_group_size(1408) == 64 and ex.best_group_size(48) == 16
    assert ex.best_group_size(40) == 0 and ex.best_group_size(1024, (64, 16)) == 64


def test_module_ingest_validation_on_cpu():
    m = ex.B200GroupedExperts.from_empty(num_experts=4, quant_format="nf4")
    with pytest.raises(ValueError, match="weight key"):
        m.load_dense_weight("w9", torch.zeros(4, 8, 8))
    with pytest.raises(ValueError, match="expected \\[4, out, in\\]"):
        m.load_dense_weight("w1", torch.zeros(3, 8, 8))
    with pytest.raises(ValueError, match="CUDA"):
        m.load_dense_weight("w1", torch.zeros(4, 128, 64))
    with pytest.raises(ValueError, match="dense shape"):
        m.load_nf4_packed_weight("w1", packed=torch.zeros(4, 1), absmax=torch.zeros(4, 1),
                                 nested_absmax=torch.zeros(4, 1), offset=torch.zeros(4), code=torch.zeros(16),
                                 nested_code=torch.zeros(256), shape=(3, 8, 8), meta=ex.Nf4Meta())
    q = ex.B200GroupedExperts.from_empty(num_experts=2, quant_format="int8")
    with pytest.raises(ValueError, match="not a power of 4"):
        q.load_quantized_weight("w1", weight_int8=torch.zeros(2, 4, 8, dtype=torch.int8),
                                weight_scale=torch.ones(2, 4, 1), group_size=8)
    with pytest.raises(ValueError, match="w1_scale"):
        q.load_quantized_weight("w1", weight_int8=torch.zeros(2, 4, 8, dtype=torch.int8),
                                weight_scale=torch.ones(2, 5, 1), group_size=0)
    q.load_quantized_weight("w1", weight_int8=torch.zeros(2, 4, 16, dtype=torch.int8),
                            weight_scale=torch.ones(2, 4, 1), group_size=16)
    assert q.w1_group_size == 16 and not q.is_fully_loaded()
    with pytest.raises(RuntimeError, match="not fully loaded"):
        q.bound_weights()


def test_tables_are_the_published_constructions():
    code = tables.nf4_code()
    assert code.shape == (16,) and code[0] == -1 and code[7] == 0 and code[15] == 1
    assert torch.all(code[1:] > code[:-1])
    dyn = tables.dynamic_map()
    assert dyn.shape == (256,) and dyn[-1] == 1.0 and torch.all(dyn[1:] >= dyn[:-1])
    from oracle import quant as oq
    assert torch.equal(code, torch.from_numpy(oq.nf4_code_table()))
    assert torch.equal(dyn, torch.from_numpy(oq.dynamic_tree_map()))
