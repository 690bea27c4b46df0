"""mirai_dispatch_plan_static (fixed in-library scratch, no workspace) against
the workspace entry point mirai_dispatch_plan.

The file name sorts last so the module runs after every other test as well as
on its own; the static scratch must give the same plans in both situations.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mirai_b200.build import build
    build()
    from mirai_b200 import _lib, ops
    return torch.device("cuda:0"), _lib, ops


def _static_plan(_lib, ops, top_indices, num_experts):
    T, k = top_indices.shape
    dev = top_indices.device
    out = [torch.full((num_experts,), -1, dtype=torch.int64, device=dev),
           torch.full((num_experts,), -1, dtype=torch.int64, device=dev),
           torch.full((num_experts,), -1, dtype=torch.int32, device=dev)]
    out += [torch.full((T * k,), -1, dtype=torch.int64, device=dev) for _ in range(3)]
    _lib.call("mirai_dispatch_plan_static", ops._ptr(top_indices), T, k, num_experts,
              *[ops._ptr(t) for t in out], ops._stream())
    return out


def _workspace_plan(ops, top_indices, num_experts):
    p = ops.dispatch_plan(top_indices, num_experts)
    return [p.counts, p.starts, p.offsets, p.sort_positions, p.sorted_token_indices, p.inverse_order]


def test_static_plan_matches_workspace_plan_on_consecutive_calls():
    dev, _lib, ops = _setup()
    gen = torch.Generator().manual_seed(11)
    cases = [(6000, 4, 64), (777, 2, 8), (33000, 2, 32)]
    results = []
    for T, k, E in cases:
        idx = torch.randint(0, E, (T, k), generator=gen).to(dev)
        results.append((_static_plan(_lib, ops, idx, E), _workspace_plan(ops, idx, E)))
    ops.check_device()
    for (got, ref), (T, k, E) in zip(results, cases):
        for g, r in zip(got, ref):
            assert torch.equal(g, r), f"plan differs for T={T} k={k} E={E}"
        assert int(got[0].sum()) == T * k


def test_static_plan_allocates_nothing():
    """After a first call on the device (which may load the library's device
    image), a static-plan call leaves the device's free memory and torch's
    allocations exactly as they were."""
    dev, _lib, ops = _setup()
    T, k, E = 20000, 4, 128
    idx = torch.randint(0, E, (T, k), generator=torch.Generator().manual_seed(3)).to(dev)
    out = [torch.empty(E, dtype=torch.int64, device=dev), torch.empty(E, dtype=torch.int64, device=dev),
           torch.empty(E, dtype=torch.int32, device=dev)] + [torch.empty(T * k, dtype=torch.int64, device=dev)
                                                             for _ in range(3)]
    args = [ops._ptr(idx), T, k, E, *[ops._ptr(t) for t in out], ops._stream()]
    _lib.call("mirai_dispatch_plan_static", *args)  # warm-up: module and symbol address
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info(dev)[0], torch.cuda.memory_allocated(dev)
    for _ in range(3):
        _lib.call("mirai_dispatch_plan_static", *args)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert torch.cuda.memory_allocated(dev) == alloc0
    ops.check_device()


def test_static_plan_checks_arguments_before_sizing():
    """An unusable expert count or token count is an argument error, not a
    scratch shortfall, and nothing is launched."""
    dev, _lib, ops = _setup()
    idx = torch.zeros((4, 2), dtype=torch.int64, device=dev)
    bufs = [torch.empty(8, dtype=torch.int64, device=dev) for _ in range(6)]
    for T, k, E in [(4, 2, 5000), (2 ** 40, 2, 8), (4, 0, 8), (-1, 2, 8)]:
        with pytest.raises(_lib.MiraiError) as err:
            _lib.call("mirai_dispatch_plan_static", ops._ptr(idx), T, k, E, *[ops._ptr(t) for t in bufs],
                      ops._stream())
        assert err.value.code == 1, str(err.value)


def test_static_plan_rejects_oversized_plans():
    dev, _lib, ops = _setup()
    limit = int(_lib.load().mirai_dispatch_plan_static_scratch_bytes())
    assert limit == 1 << 20
    E, k = 1024, 1
    T = (limit // (4 * E) + 1) * 2048  # one chunk of 2048 routes too many
    idx = torch.zeros((T, k), dtype=torch.int64, device=dev)
    out = [torch.empty(E, dtype=torch.int64, device=dev), torch.empty(E, dtype=torch.int64, device=dev),
           torch.empty(E, dtype=torch.int32, device=dev)] + [torch.empty(T * k, dtype=torch.int64, device=dev)] * 3
    with pytest.raises(_lib.MiraiError) as err:
        _lib.call("mirai_dispatch_plan_static", ops._ptr(idx), T, k, E, *[ops._ptr(t) for t in out], ops._stream())
    assert "scratch" in str(err.value) and str(limit) in str(err.value)
    # the largest plan that fits still runs and matches
    T_fit = (limit // (4 * E)) * 2048
    idx = torch.from_numpy(np.random.default_rng(5).integers(0, E, (T_fit, k))).to(dev)
    got, ref = _static_plan(_lib, ops, idx, E), _workspace_plan(ops, idx, E)
    ops.check_device()
    for g, r in zip(got, ref):
        assert torch.equal(g, r)
