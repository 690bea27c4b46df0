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


def test_token_chunk_policy_semantics():
    """MoETokenChunkPolicy's rules (token_chunking.py:25-117): size 0 disables;
    only training splits; chunks cover the tokens in order with their offsets;
    checkpointed when gradients are enabled."""
    from mirai_b200.block import TokenChunkPolicy
    calls = []

    def runner(t, s, i, off):
        calls.append((off, t.shape[0]))
        return t * 2

    x = torch.arange(10.0).reshape(10, 1)
    sc, idx = torch.ones(10, 2), torch.zeros(10, 2, dtype=torch.int64)
    assert not TokenChunkPolicy(0).enabled and TokenChunkPolicy(0).chunk_count(10) == 1
    assert TokenChunkPolicy(4).chunk_count(10) == 3
    out = TokenChunkPolicy(4).execute(x, sc, idx, runner=runner, training=True)
    assert calls == [(0, 4), (4, 4), (8, 2)] and torch.equal(out, x * 2)
    calls.clear()
    TokenChunkPolicy(4).execute(x, sc, idx, runner=runner, training=False)
    assert calls == [(0, 10)]
    calls.clear()
    xg = x.clone().requires_grad_(True)
    out = TokenChunkPolicy(3).execute(xg, sc, idx, runner=runner, training=True)
    out.sum().backward()
    assert torch.equal(xg.grad, torch.full_like(x, 2.0)) and len(calls) >= 4  # forward chunks (+ recompute)
    with pytest.raises(ValueError):
        TokenChunkPolicy(-1)
    with pytest.raises(ValueError):
        TokenChunkPolicy(4).execute(x, sc[:5], idx, runner=runner, training=True)


def test_install_on_a_reference_like_block():
    """install() puts the b200 backend on the block's kernel-backend seam and
    moves the shared expert onto SharedExpertMLP with the same parameters."""
    import torch.nn as nn
    from mirai_b200.block import SharedExpertMLP, install

    class _MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = nn.Linear(8, 16, bias=False)
            self.up_proj = nn.Linear(8, 16, bias=False)
            self.down_proj = nn.Linear(16, 8, bias=False)

    blk = types.SimpleNamespace(_mirai_moe_kernel_backend=None, shared_experts=_MLP())
    ref = blk.shared_experts.state_dict()
    install(blk)
    assert isinstance(blk._mirai_moe_kernel_backend, bk.B200MoEKernelBackend)
    assert blk._mirai_moe_kernel_backend.direct_only
    assert isinstance(blk.shared_experts, SharedExpertMLP)
    for k, v in blk.shared_experts.state_dict().items():
        assert torch.equal(v, ref[k])


def test_packed_state_entry_round_trip_on_cpu():
    """A grouped-experts entry of the reference's packed-state manifest
    (packed_state.py:331-341, 441-449): NF4 and INT8 buffers named as the
    manifest names them load into B200GroupedExperts unchanged; a missing
    tensor or a bad shape is refused with the reason."""
    from oracle import quant as oq
    E, I, H = 2, 128, 64
    rng = __import__("numpy").random.default_rng(0)
    tensors, names = {}, {}
    shapes = {"w1": (E, I, H), "w3": (E, I, H), "w2": (E, H, I)}
    for key, shp in shapes.items():
        g = oq.nf4_quantize_grouped((rng.standard_normal(shp) * 0.05).astype("float32"))
        for suffix, arr in (("nf4", g["nf4"]), ("nf4_absmax", g["absmax"]), ("nf4_nabsmax", g["nabsmax"]),
                            ("nf4_offset", g["offset"]), ("nf4_code", g["code"]), ("nf4_ncode", g["ncode"])):
            names[f"{key}_{suffix}"] = f"blocks.0.ffn.experts.{key}_{suffix}"
            tensors[names[f"{key}_{suffix}"]] = torch.from_numpy(arr.copy())
    spec = {"kind": "grouped_experts", "quant_format": "nf4", "num_experts": E, "shapes": shapes,
            "group_sizes": {"w1": 0, "w2": 0, "w3": 0}, "tensors": names,
            "nf4_meta": {"blocksize": 64, "nested_blocksize": 256, "nested_dtype": "float32",
                         "weight_dtype": "bfloat16"}}
    m = ex.B200GroupedExperts.from_packed_state(spec, tensors)
    assert m.is_fully_loaded() and m._nf4_shapes["w2"] == (E, H, I)
    for name, key in names.items():
        assert torch.equal(getattr(m, name).reshape(-1), tensors[key].reshape(-1))
    bad = dict(tensors)
    del bad[names["w3_nf4_absmax"]]
    with pytest.raises(KeyError, match="w3_nf4_absmax"):
        ex.B200GroupedExperts.from_packed_state(spec, bad)
    bad = dict(tensors)
    bad[names["w1_nf4"]] = bad[names["w1_nf4"]][:, :-2]
    with pytest.raises(ValueError, match="w1_nf4"):
        ex.B200GroupedExperts.from_packed_state(spec, bad)
    # INT8 (block-Hadamard g = 16)
    names8, t8 = {}, {}
    for key, shp in shapes.items():
        q, s, gr = oq.int8_quantize((rng.standard_normal(shp) * 0.05).astype("float32"), 16)
        names8[f"{key}_int8"], names8[f"{key}_scale"] = f"e.{key}_int8", f"e.{key}_scale"
        t8[f"e.{key}_int8"], t8[f"e.{key}_scale"] = torch.from_numpy(q), torch.from_numpy(s)
    spec8 = {"kind": "grouped_experts", "quant_format": "int8", "num_experts": E, "shapes": shapes,
             "group_sizes": {"w1": 16, "w2": 16, "w3": 16}, "tensors": names8}
    m8 = ex.B200GroupedExperts.from_packed_state(spec8, t8)
    assert m8.w1_group_size == 16 and torch.equal(m8.w2_int8, t8["e.w2_int8"])
    with pytest.raises(ValueError, match="learned rotations"):
        ex.B200GroupedExperts.from_packed_state(dict(spec8, rotations={"w1": "r"}), t8)


def test_lora_factor_pads_are_kept_until_the_factor_changes():
    """Padded adapter operands live on the factor tensor and are rebuilt only
    after the factor changes (in-place update or new storage)."""
    from mirai_b200 import ops

    p = torch.nn.Parameter(torch.randn(2, 4, 8))
    pads = ops._factor_pads(p)
    pads["b"] = "built"
    assert ops._factor_pads(p)["b"] == "built"
    with torch.no_grad():
        p.add_(1.0)  # an optimizer step
    assert "b" not in ops._factor_pads(p)
    ops._factor_pads(p)["b"] = "rebuilt"
    p.data = torch.zeros(2, 4, 8)  # new storage
    assert "b" not in ops._factor_pads(p)


def test_nf4_staging_policy(monkeypatch):
    """Which passes decode NF4 keys once into bf16 copies: training passes from
    1024 rows per expert, forward-only ones from 4096, every pass with
    "always", none with "never"; other formats are passed through."""
    from mirai_b200 import ops

    key = object.__new__(ops.NF4Tensor)  # a stand-in key: the policy only looks at its type
    decoded = []
    monkeypatch.setattr(ops, "nf4_dequantize", lambda w: decoded.append(w) or "bf16 copy")
    keys = (key, key, key)
    E = 8
    try:
        assert ops.stage_nf4(keys, 1024 * E, E, training=True) == ("bf16 copy",) * 3
        assert ops.stage_nf4(keys, 1024 * E - 1, E, training=True) == keys
        assert ops.stage_nf4(keys, 4096 * E - 1, E, training=False) == keys
        assert ops.stage_nf4(keys, 4096 * E, E, training=False) == ("bf16 copy",) * 3
        ops.set_nf4_staging("never")
        assert ops.stage_nf4(keys, 10 ** 9, E, training=True) == keys
        ops.set_nf4_staging("always")
        assert ops.stage_nf4(keys, 1, E, training=False) == ("bf16 copy",) * 3
        dense = (torch.zeros(1), torch.zeros(1), torch.zeros(1))
        assert ops.stage_nf4(dense, 10 ** 9, E, training=True) == dense
        with pytest.raises(ValueError, match="staging mode"):
            ops.set_nf4_staging("sometimes")
    finally:
        ops.set_nf4_staging("auto")
    assert len(decoded) == 9
