"""Config-tree semantics (the configgle-compatible layer)."""

from __future__ import annotations

import dataclasses
import functools
from dataclasses import KW_ONLY, field

import pytest

from priml_b200.config import Fig, InlineConfig, Makes, PartialConfig, apply_overrides, copy_tree, resolve_config


class Leaf:
    class Config(Fig["Leaf"], kw_only=False):
        width: int = -1
        _: KW_ONLY
        scale: float = 1.0

    def __init__(self, config: Config) -> None:
        self.config = config


class Parent:
    class Config(Fig["Parent"]):
        width: int = 8
        child: Leaf.Config = field(default_factory=Leaf.Config)
        children: list = field(default_factory=list)

        def finalize(self):  # noqa: ANN201
            if self.child.width == -1:
                self.child.width = self.width
            return super().finalize()

    def __init__(self, config: Config) -> None:
        self.config = config
        self.child = config.child.make()


class Special(Leaf):
    class Config(Makes["Special"], Leaf.Config):
        extra: int = 3


def test_make_builds_target_with_finalized_copy() -> None:
    cfg = Parent.Config(width=16)
    obj = cfg.make()
    assert isinstance(obj, Parent)
    assert obj.child.config.width == 16
    assert cfg.child.width == -1, "make() finalizes a copy, not the template"


def test_finalize_freezes() -> None:
    cfg = Parent.Config().finalize()
    with pytest.raises(dataclasses.FrozenInstanceError):
        cfg.width = 3
    with pytest.raises(dataclasses.FrozenInstanceError):
        cfg.child.scale = 2.0
    thawed = copy_tree(cfg)
    thawed.width = 3
    assert thawed.width == 3


def test_positional_and_kw_only_fields() -> None:
    c = Leaf.Config(4, scale=2.0)
    assert (c.width, c.scale) == (4, 2.0)
    with pytest.raises(TypeError):
        Leaf.Config(4, 2.0)  # type: ignore[misc]


def test_makes_retargets_subclass_config() -> None:
    obj = Special.Config(2).make()
    assert type(obj) is Special
    assert obj.config.extra == 3


def test_partial_and_inline_configs() -> None:
    p = PartialConfig(max, 3)
    assert isinstance(p.make(), functools.partial)
    assert p.make()(5) == 5
    i = InlineConfig(dict, a=1)
    assert i.make() == {"a": 1}
    assert i.a == 1
    i.a = 2
    assert i.make() == {"a": 2}


def test_apply_overrides_casts_to_field_type() -> None:
    cfg = Parent.Config()
    apply_overrides(cfg, ["width=32", "child.scale=0.5", "child.width=7"])
    assert cfg.width == 32 and isinstance(cfg.width, int)
    assert cfg.child.scale == 0.5
    with pytest.raises(AttributeError):
        apply_overrides(cfg, ["nope=1"])


def test_resolve_config_calls_factory() -> None:
    cfg = resolve_config("priml_b200.models.presets.tiny_lm")
    assert cfg.vocab_size == 512


def test_pformat_hides_defaults() -> None:
    text = Parent.Config(width=9).pformat()
    assert "width=9" in text
    assert "children" not in text
    full = Parent.Config(width=9).pformat(hide_default_values=False)
    assert "children" in full
