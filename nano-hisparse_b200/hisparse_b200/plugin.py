"""Routes the reference package's hot path through libhisparse.

``install(nano_hisparse)`` rebinds, inside an imported reference package, the
names its decode path looks up at call time, so that the reference's own
HybridKVCache, Model and Engine run Quest selection, the row resolver, the
miss gather and row attention on the sm_100a kernels:

  nano_hisparse.selection.quest_selection / model.quest_selection  (model.py:199-208)
  nano_hisparse.hybrid.resolve_rows                                 (hybrid.py:431-440)
  nano_hisparse.hybrid.LogicalTopK                                  (hybrid.py:406-409)
  nano_hisparse.row_kernels.MappedHost / gather_rows / attend_rows  (hybrid.py:108-111,
                                                                     447-451; attention.py:22-25)
  nano_hisparse.storage.HostStore.append                            (hybrid.py:391)

With ``indexed_residency`` (the default) it also installs
``hisparse_b200.residency``: the same residency policy, with its per-layer
scans over every page (hybrid.py:204-223, 276-277, 423-427) answered from a
per-layer index of resident pages. The policy's decisions, the storage,
model and engine are the reference's. ``uninstall`` restores the original
bindings.
"""

from __future__ import annotations

import importlib

from . import residency
from . import row_kernels as _rk
from .append import host_store_append
from .row_index import LogicalTopK, resolve_rows
from .selection import quest_selection

_BINDINGS = [
    ("selection", "quest_selection", quest_selection),
    ("model", "quest_selection", quest_selection),
    ("hybrid", "resolve_rows", resolve_rows),
    ("hybrid", "LogicalTopK", LogicalTopK),
    ("row_kernels", "MappedHost", _rk.MappedHost),
    ("row_kernels", "gather_rows", _rk.gather_rows),
    ("row_kernels", "attend_rows", _rk.attend_rows),
    ("storage", "HostStore.append", host_store_append),
]
_saved: dict = {}


def install(package, *, indexed_residency=True) -> list[str]:
    """Rebind the reference's hot-path names; returns the names rebound.

    ``package`` is the imported reference package (``import nano_hisparse``).
    The reference's row_kernels module imports Triton at import time, so the
    reference must be importable as a whole (as on a CUDA host).
    """
    done = []
    for module_name, attr, replacement in _BINDINGS:
        owner, name = _owner(package.__name__, module_name, attr)
        key = (package.__name__, module_name, attr)
        if key not in _saved:
            _saved[key] = owner.__dict__[name] if isinstance(owner, type) else getattr(owner,
                                                                                       name)
        setattr(owner, name, replacement)
        done.append(f"{module_name}.{attr}")
    if indexed_residency:
        done += residency.install(package)
    return done


def _owner(package_name, module_name, attr):
    """The object holding `attr` ("name" in the module, or "Class.name")."""
    owner = importlib.import_module(f"{package_name}.{module_name}")
    *path, name = attr.split(".")
    for part in path:
        owner = getattr(owner, part)
    return owner, name


def uninstall(package) -> None:
    residency.uninstall(package)
    for (pkg, module_name, attr), original in list(_saved.items()):
        if pkg != package.__name__:
            continue
        owner, name = _owner(pkg, module_name, attr)
        setattr(owner, name, original)
        del _saved[(pkg, module_name, attr)]
