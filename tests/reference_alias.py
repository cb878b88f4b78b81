"""pytest plugin: make the reference's module names resolve to this package.

The reference's tests import ``orchestrator``, ``compute``, ``memory``, ``runtime`` and
``api`` from its ``src`` directory; with this plugin loaded (``-p
tests.reference_alias``) those names, and every submodule under them, are this
package's modules (``metellus_b200.orchestrator`` and so on), so the reference's own
test files exercise this implementation's builder, IR, DAG, graph, fusion passes,
assembly and scheduler. Used by tests/test_reference_suite.py."""

from __future__ import annotations

import importlib
import pkgutil
import sys

for _name in ("orchestrator", "compute", "memory", "runtime", "api"):
    _mod = importlib.import_module(f"metellus_b200.{_name}")
    sys.modules[_name] = _mod
    for _sub in pkgutil.walk_packages(_mod.__path__, prefix=f"metellus_b200.{_name}."):
        sys.modules[_sub.name[len("metellus_b200."):]] = importlib.import_module(_sub.name)
