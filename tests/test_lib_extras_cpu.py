"""Library helpers, checked against the reference's own functions where it has them.

* the JSON codec, schema checker and value coercion give the reference's outputs;
* per-user directories follow the XDG variables and platform defaults;
* resource markers add aliases, timeouts and the CI skip, and refuse unknown names;
* LPIPS is zero on identical images and the video loss averages sampled frames;
* quantized activation storage keeps gradients within fp8 error.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from datetime import datetime
from enum import Enum
from pathlib import Path
from uuid import UUID

import pytest
import torch
from torch import nn

from priml_b200.testing.reference import load_reference, reference_available

needs_reference = pytest.mark.skipif(not reference_available(), reason="the reference copy is not present")


class Color(Enum):
    RED = "red"
    BLUE = "blue"


@dataclass(frozen=True)
class Leaf:
    a: int
    b: str = "x"


@dataclass(frozen=True)
class Other:
    z: float = 1.0


@dataclass(frozen=True)
class Node:
    leaf: Leaf | Other
    items: tuple[Leaf, ...] = ()
    tags: frozenset[str] = frozenset()
    meta: dict[str, int] = field(default_factory=dict)
    when: datetime | None = None
    where: Path | UUID | None = None
    color: Color = Color.RED
    raw: bytes = b""
    pair: tuple[int, str] = (0, "")


NODE = Node(leaf=Other(2.5), items=(Leaf(1), Leaf(2, "y")), tags=frozenset({"b", "a"}), meta={"k": 3},
            when=datetime(2024, 1, 2, 3, 4, 5), where=UUID(int=5), color=Color.BLUE, raw=b"\x00\x01",
            pair=(4, "q"))  # fmt: skip

SCHEMAS = [
    ({"type": "object", "properties": {"a": {"type": "integer", "minimum": 0}}, "required": ["a", "b"],
      "additionalProperties": False}, {"a": -1, "c": 2}),
    ({"type": ["array", "string"], "items": {"enum": [1, "x"]}}, [1, 2, "x"]),
    ({"type": "number", "maximum": 3}, True),
    ({"type": "object", "additionalProperties": {"type": "string"}}, {"k": 1, "j": "ok"}),
    ({"type": "object", "properties": {"n": {"type": "object", "properties": {"m": {"type": "null"}}}}},
     {"n": {"m": 0}}),
]  # fmt: skip

VALUES = ["false", "yes", "maybe", "", " 7 ", "3.7", 0, 2, 2.9, True, None, [1], {"a": 1}]


def test_codec_round_trip_and_schema_error() -> None:
    from priml_b200.lib.custom_json import JsonCodec, SchemaError, dataclass_from_json, dataclass_to_json

    data = dataclass_to_json(NODE)
    assert data["leaf"] == {"__type__": "Other", "z": 2.5}
    assert data["where"] == {"__scalar__": "UUID", "__value__": str(UUID(int=5))}
    assert dataclass_from_json(Node, data) == NODE
    with pytest.raises(SchemaError, match="zz"):
        dataclass_from_json(Leaf, {"a": 1, "zz": 2})
    assert dataclass_from_json(Leaf, {"a": "4", "b": 5}) == Leaf(4, "5")

    @dataclass(frozen=True)
    class Mixed(JsonCodec):
        leaf: Leaf

    assert Mixed.from_json(Mixed(Leaf(3)).to_json()) == Mixed(Leaf(3))


@needs_reference
def test_codec_and_helpers_match_reference() -> None:
    load_reference()
    import priml.lib.custom_json as ref

    import priml_b200.lib.custom_json as ours

    assert ours.dataclass_to_json(NODE) == ref.dataclass_to_json(NODE)
    assert ours.dataclass_from_json(Node, ref.dataclass_to_json(NODE)) == NODE
    assert ref.dataclass_from_json(Node, ours.dataclass_to_json(NODE)) == NODE
    for schema, value in SCHEMAS:
        assert ours.validate_json_schema(schema, value) == ref.validate_json_schema(schema, value)
    for v in VALUES:
        assert ours.bool_val(v, True) == ref.bool_val(v, True), v
        assert ours.int_val(v, -1) == ref.int_val(v, -1), v
        assert ours.float_val(v, -1.0) == ref.float_val(v, -1.0), v
        assert ours.str_val(v, "d") == ref.str_val(v, "d"), v
        assert ours.list_val(v) == ref.list_val(v), v
        assert ours.dict_val(v) == ref.dict_val(v), v
        assert ours.datetime_val(v) == ref.datetime_val(v), v
    nested = {"a": [1, {"b": (2, 3)}], "c": {"d": None}}
    assert ours.json_unfreeze(ours.json_freeze(nested)) == ref.json_unfreeze(ref.json_freeze(nested))
    assert ours.dicts_val([{"a": 1}, {}, 3]) == ref.dicts_val([{"a": 1}, {}, 3])


def test_userdirs_follow_xdg_and_platform(monkeypatch: pytest.MonkeyPatch) -> None:
    from priml_b200.lib import userdirs

    home = Path.home()
    for var in ("XDG_DATA_HOME", "XDG_CONFIG_HOME", "XDG_CACHE_HOME", "XDG_STATE_HOME", "LOCALAPPDATA"):
        monkeypatch.delenv(var, raising=False)
    assert userdirs.cache_dir(platform="linux") == home / ".cache"
    assert userdirs.state_dir(platform="linux") == home / ".local" / "state"
    assert userdirs.cache_dir(platform="darwin") == home / "Library" / "Caches"
    assert userdirs.config_dir(platform="darwin") == home / "Library" / "Application Support"
    assert userdirs.data_dir(platform="win32") == home / "AppData" / "Local"
    monkeypatch.setenv("XDG_CACHE_HOME", "rel/cache")
    monkeypatch.setenv("XDG_CONFIG_HOME", "")
    assert userdirs.cache_dir(platform="darwin") == Path("rel/cache")  # relative and honoured on macOS
    assert userdirs.config_dir(platform="linux") == home / ".config"  # empty means unset
    monkeypatch.setenv("LOCALAPPDATA", "C:/L")
    assert userdirs.cache_dir(platform="win32") == Path("C:/L")


@needs_reference
def test_userdirs_match_reference(monkeypatch: pytest.MonkeyPatch) -> None:
    load_reference()
    from priml.lib import userdirs as ref

    from priml_b200.lib import userdirs as ours

    monkeypatch.setenv("XDG_STATE_HOME", "/x/state")
    monkeypatch.delenv("XDG_DATA_HOME", raising=False)
    for plat in ("linux", "darwin", "win32"):
        for fn in ("data_dir", "config_dir", "cache_dir", "state_dir"):
            assert getattr(ours, fn)(platform=plat) == getattr(ref, fn)(platform=plat), (plat, fn)


class _Item:
    """A collected test as the marker hook sees it."""

    def __init__(self, *names: str) -> None:
        self.marks = [getattr(pytest.mark, n).mark for n in names]

    def iter_markers(self, name: str | None = None):  # noqa: ANN201
        return iter([m for m in self.marks if name is None or m.name == name])

    def get_closest_marker(self, name: str) -> pytest.Mark | None:
        return next(self.iter_markers(name), None)

    def add_marker(self, marker, *, append: bool = True) -> None:  # noqa: ANN001
        self.marks.append(marker.mark if hasattr(marker, "mark") else getattr(pytest.mark, marker).mark)


def test_resource_markers(monkeypatch: pytest.MonkeyPatch) -> None:
    from priml_b200.lib.testing.resource_markers import RESOURCES, apply_resource_markers, resource_marker_timeout

    monkeypatch.delenv("CI", raising=False)
    item = _Item("gpu_multi", "compute_distributed")
    apply_resource_markers([item], resource_markers=RESOURCES)
    names = [m.name for m in item.marks]
    assert "cuda" in names and "slow" in names and "skip" not in names
    assert item.get_closest_marker("timeout").args == (600,)
    apply_resource_markers([item], resource_markers=RESOURCES)  # a second conftest binding adds nothing
    assert sorted(m.name for m in item.marks) == sorted(names)
    assert resource_marker_timeout("network_wandb") == 180

    monkeypatch.setenv("CI", "1")
    ci_item = _Item("gpu_torch_cuda")
    apply_resource_markers([ci_item], resource_markers=RESOURCES)
    assert ci_item.get_closest_marker("skip") is not None
    monkeypatch.setenv("RUN_INTEGRATION", "1")
    opted = _Item("gpu_torch_cuda")
    apply_resource_markers([opted], resource_markers=RESOURCES)
    assert opted.get_closest_marker("skip") is None

    with pytest.raises(pytest.UsageError, match="gpu_typo"):
        apply_resource_markers([_Item("gpu_typo")], resource_markers=RESOURCES)


def test_lpips_identity_symmetry_and_video_loss() -> None:
    from priml_b200.loss import LPIPS, LPIPSLoss
    from priml_b200.loss.lpips import remap_lpips_checkpoint

    torch.manual_seed(0)
    metric = LPIPS("alex")
    a, b = torch.rand(2, 3, 64, 64) * 2 - 1, torch.rand(2, 3, 64, 64) * 2 - 1
    assert metric(a, a).abs().max() == 0
    d = metric(a, b)
    assert d.shape == (2, 1, 1, 1) and (d > 0).all()
    torch.testing.assert_close(d, metric(b, a))
    assert set(remap_lpips_checkpoint({"lin0.model.1.weight": torch.ones(1, 64, 1, 1), "other": torch.zeros(1)})) == {
        "lins.0.weight"}

    calls = []

    def fake(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        calls.append(x.shape)
        return (x - y).abs().mean(dim=(1, 2, 3), keepdim=True)

    loss = LPIPSLoss(LPIPSLoss.Config(max_num_random_frames=3), criterion=fake)
    x = torch.randn(2, 3, 5, 8, 8)
    out = loss(None, x=x, xhat=x + 1.0)["loss"]
    assert out.shape == (2,) and calls == [torch.Size([6, 3, 8, 8])]
    torch.testing.assert_close(out, torch.ones(2))


def test_quantized_activation_storage_keeps_gradients() -> None:
    from priml_b200.train import QuantizedActivationStorage, QuantizedModuleActivationStorage

    torch.manual_seed(0)

    def net() -> nn.Module:
        torch.manual_seed(1)
        return nn.Sequential(nn.Conv2d(3, 8, 3, padding=1), nn.ReLU(), nn.Flatten(), nn.Linear(8 * 16 * 16, 4))

    x = torch.randn(4, 3, 16, 16)
    plain, per_module, hooked = net(), net(), net()
    QuantizedModuleActivationStorage.Config(module_types=(nn.Conv2d, nn.Linear), min_size=16).make()(per_module)
    QuantizedActivationStorage.Config(min_size=16).make()(hooked)
    for m in (plain, per_module, hooked):
        m(x).square().sum().backward()
    for other in (per_module, hooked):
        for (name, p), q in zip(plain.named_parameters(), other.parameters(), strict=True):
            rel = float((p.grad - q.grad).norm() / p.grad.norm().clamp_min(1e-12))
            assert rel < 0.08, (name, rel)  # e4m3 keeps 3 mantissa bits
    with pytest.raises(ValueError, match="not supported"):
        QuantizedModuleActivationStorage.Config(module_types=(nn.GRU,)).make()
