"""Shared-memory lifetime analysis, alias planning and the fusion budget
(reference: src/orchestrator/aliasing.py:44-471).

The algorithm is the reference's — lifetimes over top-level fragment indices
(recursing into ``sub_fragments``), birth-order greedy slot packing that minimises
slot growth, then a rewrite that replaces multi-tenant slots with one flat storage
array and re-types it for each tenant with an ``AliasFragment`` (plus a barrier when
the seam has none).

The cap is re-derived for B200: the reference's 32 KB Apple threadgroup limit becomes
the sm_100a per-block opt-in maximum of 227 KB (232,448 bytes,
cudaDevAttrMaxSharedMemoryPerBlockOptin), so fusion decisions are made against the
real B200 budget. Kernels that reserve shared memory of their own (mbarriers, TMEM
address slot) report it through ``CodegenContext.static_smem_bytes``, which counts
against the same cap.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Iterable

from metellus_b200.compute.fragments import AliasFragment, TgmemAccess, parse_smem_decl
from metellus_b200.orchestrator.kernel_group import KernelGroup
from metellus_b200.runtime.program import Kernel

SM100_SMEM_OPTIN_BYTES = 232_448
TGMEM_CAP_BYTES = SM100_SMEM_OPTIN_BYTES


class TgmemOverflowError(RuntimeError):
    """A kernel's shared-memory footprint cannot fit under ``TGMEM_CAP_BYTES``."""


@dataclass(frozen=True)
class TgmemLifetime:
    name: str
    birth: int
    death: int
    size_floats: int
    shape: tuple[int, int]


def _walk_accesses(fragment: object) -> Iterable[TgmemAccess]:
    yield from getattr(fragment, "tgmem_accesses", ())
    for sub in getattr(fragment, "sub_fragments", ()):
        yield from _walk_accesses(sub)


def compute_lifetimes(kernel: Kernel) -> tuple[TgmemLifetime, ...]:
    order: list[str] = []
    birth: dict[str, int] = {}
    death: dict[str, int] = {}
    size: dict[str, int] = {}
    shape: dict[str, tuple[int, int]] = {}
    for idx, frag in enumerate(kernel.fragments):
        for a in _walk_accesses(frag):
            if a.name not in birth:
                order.append(a.name)
                birth[a.name] = idx
                size[a.name] = a.size_floats
                shape[a.name] = a.shape
            death[a.name] = idx
            if a.size_floats > size[a.name]:
                size[a.name] = a.size_floats
                shape[a.name] = a.shape
    return tuple(TgmemLifetime(n, birth[n], death[n], size[n], shape[n]) for n in order)


def compute_group_lifetimes(group: KernelGroup) -> tuple[TgmemLifetime, ...]:
    return compute_lifetimes(group.kernel)


@dataclass(frozen=True)
class FusionBudget:
    """Post-alias shared-memory footprint of one kernel."""

    n_slots: int
    size_floats: int
    static_bytes: int = 0

    @property
    def size_bytes(self) -> int:
        return self.size_floats * 4 + self.static_bytes


@dataclass(frozen=True)
class AliasSlot:
    name: str
    tenants: tuple[str, ...]
    size_floats: int
    shape: tuple[int, int]


@dataclass(frozen=True)
class AliasMap:
    slots: tuple[AliasSlot, ...]

    @property
    def name_to_slot(self) -> dict[str, str]:
        return {t: s.name for s in self.slots for t in s.tenants}

    @property
    def total_size_floats(self) -> int:
        return sum(s.size_floats for s in self.slots)

    @property
    def n_slots(self) -> int:
        return len(self.slots)


def compute_alias_map(lifetimes: tuple[TgmemLifetime, ...]) -> AliasMap:
    """Birth-order greedy packing; a lifetime joins the disjoint slot with the least
    growth, then the smallest current size, then the most recently freed last tenant
    (aliasing.py:209-289)."""
    slots: list[list[TgmemLifetime]] = []
    sizes: list[int] = []
    for lt in sorted(lifetimes, key=lambda x: (x.birth, x.death)):
        best, best_key = None, None
        for i, tenants in enumerate(slots):
            last = tenants[-1]
            if last.death >= lt.birth:
                continue
            cur = sizes[i]
            key = (max(0, lt.size_floats - cur), cur, -last.death)
            if best_key is None or key < best_key:
                best, best_key = i, key
        if best is None:
            slots.append([lt])
            sizes.append(lt.size_floats)
        else:
            slots[best].append(lt)
            sizes[best] = max(sizes[best], lt.size_floats)
    return AliasMap(tuple(AliasSlot(t[0].name, tuple(x.name for x in t), s, t[0].shape)
                          for t, s in zip(slots, sizes)))


def compute_budget(lifetimes: tuple[TgmemLifetime, ...], static_bytes: int = 0) -> FusionBudget:
    m = compute_alias_map(lifetimes)
    return FusionBudget(n_slots=m.n_slots, size_floats=m.total_size_floats, static_bytes=static_bytes)


def compute_group_budget(group: KernelGroup) -> FusionBudget:
    return compute_budget(compute_lifetimes(group.kernel), group.kernel.ctx.static_smem_bytes)


def compute_group_alias_map(group: KernelGroup) -> AliasMap:
    return compute_alias_map(compute_lifetimes(group.kernel))


def _is_barrier(fragment: object) -> bool:
    return getattr(fragment, "is_tgmem_barrier", False) is True


def _storage_name(owner: str) -> str:
    return f"_{owner}_storage"


def apply_alias_map(kernel: Kernel, alias_map: AliasMap) -> Kernel:
    """Rewrite ``kernel`` to the plan (aliasing.py:340-453): single-tenant slots keep
    their decl; multi-tenant slots get one flat storage decl and an AliasFragment per
    tenant, placed after the latest barrier in the seam (or with its own barrier)."""
    if not alias_map.slots:
        return kernel
    by_name = {lt.name: lt for lt in compute_lifetimes(kernel)}
    inserts: dict[int, list[AliasFragment]] = {}
    new_decls_tail: list[str] = []
    dropped: set[str] = set()
    kept: set[str] = set()
    for slot in alias_map.slots:
        if len(slot.tenants) == 1:
            kept.add(slot.name)
            continue
        storage = _storage_name(slot.name)
        new_decls_tail.append(f"smem float {storage}[{slot.size_floats}];")
        dropped.update(slot.tenants)
        prev_death = -1
        for i, tenant in enumerate(slot.tenants):
            lt = by_name[tenant]
            if i == 0:
                at, pre = -1, True
            else:
                bar = None
                for j in range(prev_death + 1, lt.birth):
                    if _is_barrier(kernel.fragments[j]):
                        bar = j
                at, pre = (bar, True) if bar is not None else (lt.birth - 1, False)
            inserts.setdefault(at, []).append(AliasFragment(storage, tenant, lt.shape, pre))
            prev_death = lt.death
    frags: list = list(inserts.get(-1, ()))
    for i, f in enumerate(kernel.fragments):
        frags.append(f)
        frags.extend(inserts.get(i, ()))
    decls: list[str] = []
    for d in kernel.ctx.threadgroup_decls:
        name, _ = parse_smem_decl(d)
        if name in kept:
            decls.append(d)
        elif name not in dropped:
            raise ValueError(
                f"apply_alias_map: shared decl {d!r} declares {name!r}, which is in no alias "
                "slot — lifetime analysis missed a shared-memory object"
            )
    decls.extend(new_decls_tail)
    return Kernel(tuple(frags), dataclasses.replace(kernel.ctx, threadgroup_decls=tuple(decls)))


def apply_group_alias_map(group: KernelGroup, alias_map: AliasMap) -> KernelGroup:
    return dataclasses.replace(group, kernel=apply_alias_map(group.kernel, alias_map))


def alias_group(group: KernelGroup) -> KernelGroup:
    """Lifetimes -> plan -> rewrite for one group (aliasing.py:463-471)."""
    return apply_group_alias_map(group, compute_alias_map(compute_lifetimes(group.kernel)))
