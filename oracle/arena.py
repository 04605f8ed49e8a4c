"""Oracle restatement of the arena planner, src/engine/arena.ts:57-172.

TEST INFRASTRUCTURE ONLY: checks the product's C++ planner.
"""
from __future__ import annotations

from .arch import Architecture, op_inputs


def tensor_elements(s) -> int:
    """tensorElements, src/model/layout.ts:23-25 (vec4 count)."""
    return s.h * s.w * (s.c // 4)


def plan_arena(arch: Architecture, exclude: set):
    """planArena, arena.ts:57-128. Returns (buffer_sizes_vec4, assignment, total_bytes, naive_bytes)."""
    last_read = {}
    for i, op in enumerate(arch.ops):
        for t in op_inputs(op):
            last_read[t] = i
    sizes, free, assignment, occupant = [], [], {}, {}
    for i, op in enumerate(arch.ops):
        out = op.out
        if out not in exclude and out not in assignment:
            need = tensor_elements(arch.tensors[out])
            chosen, chosen_size = -1, float("inf")
            for b in range(len(sizes)):
                if free[b] and sizes[b] >= need and sizes[b] < chosen_size:
                    chosen, chosen_size = b, sizes[b]
            if chosen == -1:
                grow, grow_size = -1, -1
                for b in range(len(sizes)):
                    if free[b] and sizes[b] > grow_size:
                        grow, grow_size = b, sizes[b]
                if grow == -1:
                    chosen = len(sizes)
                    sizes.append(need)
                    free.append(False)
                else:
                    chosen = grow
                    sizes[grow] = need
            free[chosen] = False
            assignment[out] = chosen
            occupant[chosen] = out
        for t in op_inputs(op):
            if last_read.get(t) == i:
                b = assignment.get(t)
                if b is not None and occupant.get(b) == t:
                    free[b] = True
    total = sum(n * 16 for n in sizes)
    naive = sum(tensor_elements(s) * 16 for n, s in arch.tensors.items() if n not in exclude)
    return sizes, assignment, total, naive


def validate_arena(arch: Architecture, sizes, assignment, exclude: set) -> None:
    """validateArena, arena.ts:134-172. Raises ValueError on a violation."""
    first_write, last_read = {}, {}
    for i, op in enumerate(arch.ops):
        first_write.setdefault(op.out, i)
        for t in op_inputs(op):
            last_read[t] = i
    names = [n for n in arch.tensors if n not in exclude]
    for a in names:
        for b in names:
            if a >= b or assignment.get(a) != assignment.get(b):
                continue
            a0 = first_write.get(a, 0)
            a1 = last_read.get(a, a0)
            b0 = first_write.get(b, 0)
            b1 = last_read.get(b, b0)
            if a0 <= b1 and b0 <= a1:
                raise ValueError(f"arena: {a} [{a0}..{a1}] and {b} [{b0}..{b1}] overlap in buffer {assignment.get(a)}")
    for n in names:
        b = assignment.get(n)
        if b is None:
            raise ValueError(f"arena: {n} was never assigned a buffer")
        need = tensor_elements(arch.tensors[n])
        if sizes[b] < need:
            raise ValueError(f"arena: buffer {b} holds {sizes[b]} but {n} needs {need}")
