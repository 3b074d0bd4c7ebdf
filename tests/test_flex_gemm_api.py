"""The drop-in flex_gemm package exposes the reference operator package's API (recorded in
tests/golden/flex_gemm_api.json by tests/golden/make_flex_api.py): same names, same constructor / forward / function
parameters with the same kinds and defaults (extra parameters only keyword-only with defaults), a superset of
NeighborCache's public members; registers under the import name; refuses CPU tensors and gradients.  CPU only."""
import inspect
import json
import sys
from pathlib import Path

import pytest
import torch

API = json.loads((Path(__file__).parent / "golden" / "flex_gemm_api.json").read_text())


def _sig(fn):
    return {p.name: (p.kind.name, None if p.default is inspect.Parameter.empty else repr(p.default))
            for p in inspect.signature(fn).parameters.values()}


def _check(ours, ref_list, where):
    for name, kind, default in ref_list:
        assert name in ours, f"{where}: missing parameter {name}"
        assert ours[name] == (kind, default), f"{where}: {name} {ours[name]} != {(kind, default)}"
    extra = set(ours) - {r[0] for r in ref_list}
    for name in extra:
        kind, default = ours[name]
        assert kind == "KEYWORD_ONLY" and default is not None, f"{where}: extra parameter {name} must be optional"


def test_nn_and_ops_names():
    from promptmoge_b200.flex_gemm import nn, ops
    assert set(API["nn_all"]) <= set(nn.__all__)
    assert set(API["ops_all"]) <= set(ops.__all__)


@pytest.mark.parametrize("name", sorted(API["nn"]))
def test_module_signatures(name):
    from promptmoge_b200.flex_gemm import nn
    cls = getattr(nn, name)
    _check(_sig(cls.__init__), API["nn"][name]["init"], f"{name}.__init__")
    _check(_sig(cls.forward), API["nn"][name]["forward"], f"{name}.forward")


@pytest.mark.parametrize("name", sorted(API["ops"]))
def test_ops_signatures(name):
    from promptmoge_b200.flex_gemm import ops
    obj = getattr(ops, name)
    ref = API["ops"][name]
    if ref["class"]:
        _check(_sig(obj.__init__), ref["init"], f"{name}.__init__")
        assert set(ref["members"]) <= {n for n in dir(obj) if not n.startswith("_")}
    else:
        _check(_sig(obj), ref["sig"], name)


def test_parameters_match_reference_shapes_and_init():
    from promptmoge_b200.flex_gemm import nn
    torch.manual_seed(0)
    conv = nn.SubmanifoldConv3d(16, 32, 3, algorithm="implicit_gemm")
    assert conv.weight.shape == (32, 3, 3, 3, 16) and conv.bias.shape == (32,)
    assert isinstance(conv.weight, torch.nn.Parameter)
    bound = 1.0 / (16 * 27) ** 0.5
    assert float(conv.bias.abs().max()) <= bound
    assert nn.SparsePool3d(2, stride=2, reduce="mean").stride == (2, 2, 2)
    assert nn.SparseUpsample3d(2, mode="nearest").scale_factor == (2, 2, 2)


def test_install_registers_import_name(monkeypatch):
    import promptmoge_b200.flex_gemm as pkg
    monkeypatch.delitem(sys.modules, "flex_gemm", raising=False)
    monkeypatch.delitem(sys.modules, "flex_gemm.nn", raising=False)
    monkeypatch.delitem(sys.modules, "flex_gemm.ops", raising=False)
    pkg.install()
    from flex_gemm.nn import SubmanifoldConv3d
    from flex_gemm.ops import NeighborCache
    assert SubmanifoldConv3d is pkg.nn.SubmanifoldConv3d and NeighborCache is pkg.ops.NeighborCache


def test_kernel_delta_order():
    from promptmoge_b200.flex_gemm.ops import make_conv_kernel_delta
    from oracle import structure as ost
    d = make_conv_kernel_delta((3, 3, 3), (1, 1, 1), batch_dims=1)
    assert d.tolist() == ost.kernel_delta().tolist()


def test_cpu_tensors_are_refused():
    """No silent CPU path: host tensors raise before any compute."""
    from promptmoge_b200.flex_gemm.ops import build_submanifold_cache
    coords = torch.zeros((4, 4), dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        build_submanifold_cache(coords, (1, 4, 4, 4), (3, 3, 3))


def test_unsupported_configurations_raise():
    from promptmoge_b200.flex_gemm.ops import build_pool_cache, build_submanifold_cache
    c = torch.zeros((4, 4), dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        build_submanifold_cache(c, (1, 4, 4, 4), (5, 5, 5))
    with pytest.raises(AssertionError):
        build_pool_cache(c, (1, 4, 4, 4), (2, 2, 2), (1, 1, 1), (0, 0, 0))
