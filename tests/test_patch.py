"""Kernel-pack mechanics of specdec_b200.kernels.patch (specdec/kernels/patch.py:139-173):
which entry points each pack replaces, restore, unknown packs, current_pack.  CPU only:
nothing here calls a kernel."""

from __future__ import annotations

import importlib
import os
import sys
import types

import pytest

from specdec_b200.kernels import patch


def _fake_engine():
    m = types.ModuleType("fake_model_self")

    class RMSNORM:
        def forward(self, x):
            return "rms"

    class MLP:
        def forward(self, x):
            return "mlp"

    class SelfAttention:
        def forward(self, x, cos, sin, cache=None):
            return "attn", cache

    m.RMSNORM, m.MLP, m.SelfAttention = RMSNORM, MLP, SelfAttention
    m.apply_rope = lambda x, cos, sin: "rope"
    return m


@pytest.fixture()
def fake():
    m = _fake_engine()
    patch.set_target(m)
    yield m
    patch.set_target(None)


PARTS = {
    "rms": lambda m: m.RMSNORM.forward,
    "rope": lambda m: m.apply_rope,
    "swiglu": lambda m: m.MLP.forward,
    "attn": lambda m: m.SelfAttention.forward,
}
EXPECT = {
    "torch": set(),
    "elementwise": {"rms", "rope", "swiglu"},
    "attention": {"attn"},
    "all": {"rms", "rope", "swiglu", "attn"},
}


@pytest.mark.parametrize("pack", sorted(EXPECT))
def test_pack_replaces_exactly_its_entry_points(fake, pack):
    orig = {k: f(fake) for k, f in PARTS.items()}
    assert patch.install(pack) == pack
    assert patch.current_pack() == pack
    for part, get in PARTS.items():
        replaced = get(fake) is not orig[part]
        assert replaced == (part in EXPECT[pack]), (pack, part)
    patch.restore()
    assert patch.current_pack() == "torch"
    for part, get in PARTS.items():
        assert get(fake) is orig[part]


def test_packs_do_not_stack(fake):
    orig_rms = fake.RMSNORM.forward
    patch.install("elementwise")
    patch.install("attention")  # starts from the originals again
    assert fake.RMSNORM.forward is orig_rms
    patch.restore()


def test_unknown_pack_raises_value_error(fake):
    with pytest.raises(ValueError):
        patch.install("fast")
    assert patch.current_pack() == "torch"


def test_restore_without_install_is_a_no_op(fake):
    orig = fake.SelfAttention.forward
    patch.restore()
    assert fake.SelfAttention.forward is orig
    assert patch.current_pack() == "torch"


def test_reference_engine_classes_when_importable(monkeypatch):
    """The default target is the reference engine module; patch it when it imports here."""
    try:
        root = os.environ.get("REFERENCE_ROOT")
        if not root:
            pytest.skip("REFERENCE_ROOT is not set")
        monkeypatch.syspath_prepend(root)
        m = importlib.import_module("specdec.engine.model_self")
    except Exception:
        pytest.skip("reference engine not importable in this environment")
    patch.set_target(None)
    try:
        orig = m.SelfAttention.forward
        patch.install("all")
        assert m.SelfAttention.forward is not orig
        assert m.RMSNORM.forward.__module__ == "specdec_b200.kernels.patch"
        patch.restore()
        assert m.SelfAttention.forward is orig
    finally:
        patch.restore()
        patch.set_target(None)
        for name in [n for n in sys.modules if n == "specdec" or n.startswith("specdec.")]:
            del sys.modules[name]
