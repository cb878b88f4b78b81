"""Extra input buffers pulled in by prologue / epilogue chains (reference:
assembly/extras.py:27-41): deduplicated by storage owner (``buffer_key``) so an
aliased view binds its owner, appended after the template's base slots."""

from __future__ import annotations

import re
from dataclasses import dataclass, field

from metellus_b200.orchestrator.ir import Tensor


def pname(key: str) -> str:
    """C identifier of the kernel parameter bound to buffer ``key`` (prefixed so a
    tensor named like a dim or a local, e.g. ``N`` or ``row``, cannot collide)."""
    return "g_" + re.sub(r"[^0-9A-Za-z_]", lambda m: f"_{ord(m.group(0)):02x}", key)


def param_decl(key: str, *, writable: bool = False) -> str:
    return f"float* {pname(key)}" if writable else f"const float* __restrict__ {pname(key)}"


@dataclass
class Extras:
    buffers: list[str] = field(default_factory=list)
    bindings: list[str] = field(default_factory=list)
    batch_strides: list[int] = field(default_factory=list)
    seen: set[str] = field(default_factory=set)
    base_slots_by_key: dict[str, int] = field(default_factory=dict)

    def add_tensor(self, t: Tensor, base_slot: int) -> int:
        key = t.buffer_key
        if key in self.base_slots_by_key:
            return self.base_slots_by_key[key]
        if key in self.seen:
            return self.bindings.index(key) + base_slot
        slot = base_slot + len(self.bindings)
        self.buffers.append(param_decl(key))
        self.bindings.append(key)
        self.batch_strides.append(t.batch_stride if len(t.shape) == 3 else 0)
        self.seen.add(key)
        return slot
