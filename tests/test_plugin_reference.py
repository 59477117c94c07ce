"""The plugin against the REAL reference package (CPU; skipped where the
reference checkout is absent, e.g. on a GPU box).

plugin.install rebinds names inside an imported nano_hisparse. For that to be
a drop-in, every rebound name must exist where the reference looks it up, the
reference's callers must look it up at call time (a module global or a lazy
import, not a reference captured at import), and every replacement must
accept exactly the arguments the original accepts. Checked here on the
reference itself:
  selection.py:69 / model.py:16,201   quest_selection
  row_index.py:62 / hybrid.py:16,431  resolve_rows
  row_index.py:15-51 / hybrid.py:408  LogicalTopK
  row_kernels.py:10 / hybrid.py:109   MappedHost
  row_kernels.py:58 / hybrid.py:449   gather_rows
  row_kernels.py:116 / attention.py:23 attend_rows
  storage.py:258 / hybrid.py:391      HostStore.append
"""

from __future__ import annotations

import dataclasses
import importlib
import inspect
import os
import sys
from pathlib import Path

import pytest

REFERENCE = Path(os.environ.get("NANO_HISPARSE_REFERENCE", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REFERENCE / "nano_hisparse").is_dir(),
                                reason="reference checkout not available")


@pytest.fixture(scope="module")
def reference():
    sys.dont_write_bytecode = True  # the checkout may be read-only
    sys.path.insert(0, str(REFERENCE))
    try:
        yield importlib.import_module("nano_hisparse")
    finally:
        sys.path.remove(str(REFERENCE))


def _call_shape(fn, bound_method=False):
    """(name, kind, default) of every parameter; annotations are not part of
    the calling contract, nor is the name of a method's bound first argument."""
    params = list(inspect.signature(fn).parameters.values())
    shape = [(p.name, p.kind, p.default) for p in params]
    if bound_method:
        shape[0] = ("<bound>", shape[0][1], shape[0][2])
    return shape


def _original(package, module_name, attr):
    from hisparse_b200 import plugin

    owner, name = plugin._owner(package.__name__, module_name, attr)
    return owner.__dict__[name] if isinstance(owner, type) else getattr(owner, name)


def test_every_rebound_name_exists_with_the_same_call_shape(reference):
    from hisparse_b200 import plugin

    assert plugin._BINDINGS, "no bindings"
    for module_name, attr, replacement in plugin._BINDINGS:
        original = _original(reference, module_name, attr)
        method = "." in attr
        assert _call_shape(replacement, method) == _call_shape(original, method), \
            f"{module_name}.{attr}"


def test_value_types_keep_the_reference_fields(reference):
    from hisparse_b200 import row_index, selection

    ref_index = importlib.import_module("nano_hisparse.row_index")
    for name in ("LogicalTopK", "RowPlan"):
        ours = [f.name for f in dataclasses.fields(getattr(row_index, name))]
        theirs = [f.name for f in dataclasses.fields(getattr(ref_index, name))]
        assert ours == theirs, name
    assert hasattr(row_index.LogicalTopK, "from_selection")
    assert hasattr(row_index.LogicalTopK, "validate")
    ref_sel = importlib.import_module("nano_hisparse.selection").Selection
    for member in ("positions", "length", "page_size", "source", "pages", "from_tokens",
                   "from_pages"):
        assert hasattr(ref_sel, member) or member in ref_sel.__dataclass_fields__, member
        assert hasattr(selection.Selection, member) or member in selection.Selection.__slots__ \
            or f"_{member}" in selection.Selection.__slots__, member
    for ctor in ("from_tokens", "from_pages"):
        assert _call_shape(getattr(selection.Selection, ctor)) == \
            _call_shape(getattr(ref_sel, ctor)), ctor


def test_reference_callers_look_the_names_up_at_call_time(reference):
    """Each caller names the rebound function through its module's globals or
    a lazy import inside the function body, so a rebinding after import is
    seen by the next call."""
    mods = {m: importlib.import_module(f"nano_hisparse.{m}")
            for m in ("model", "hybrid", "attention", "selection", "row_kernels", "storage")}
    callers = [
        (mods["model"].Model.decode, "quest_selection", "model"),
        (mods["hybrid"].HybridKVCache.resolve, "resolve_rows", "hybrid"),
        (mods["hybrid"].HybridKVCache.attention, "LogicalTopK", "hybrid"),
        (mods["hybrid"].HybridKVCache.__init__, "MappedHost", None),     # lazy import
        (mods["hybrid"].HybridKVCache.resolve, "gather_rows", None),     # lazy import
        (mods["attention"].row_attention, "attend_rows", None),          # lazy import
    ]
    for fn, name, global_module in callers:
        code = inspect.unwrap(fn).__code__  # past decorators such as torch.no_grad
        names = set(code.co_names)
        for const in code.co_consts:  # nested code objects (comprehensions, closures)
            if inspect.iscode(const):
                names |= set(const.co_names)
        assert name in names, f"{fn.__qualname__} does not name {name}"
        if global_module is not None:
            # a module global: the rebinding target is that module's attribute
            assert hasattr(mods[global_module], name)
    # HostStore.append is called as a bound method (hybrid.py:391)
    assert "append" in mods["hybrid"].HybridKVCache.write.__code__.co_names


def test_install_and_uninstall_on_the_reference(reference):
    from hisparse_b200 import plugin

    originals = {(m, a): _original(reference, m, a) for m, a, _ in plugin._BINDINGS}
    bound = plugin.install(reference)
    try:
        indexed = ["DeviceAllocator.bind", "DeviceAllocator.release", "DeviceAllocator.unpin",
                   "HybridKVCache._historical_pages", "HybridKVCache._unpin_clean_pages",
                   "HybridKVCache.update_residency", "HybridKVCache.resolve"]
        assert sorted(bound) == sorted([f"{m}.{a}" for m, a, _ in plugin._BINDINGS] + indexed)
        for module_name, attr, replacement in plugin._BINDINGS:
            assert _original(reference, module_name, attr) is replacement
    finally:
        plugin.uninstall(reference)
    for (module_name, attr), value in originals.items():
        assert _original(reference, module_name, attr) is value
    hybrid = importlib.import_module(f"{reference.__name__}.hybrid")
    assert hybrid.HybridKVCache.update_residency.__module__ == f"{reference.__name__}.hybrid"
