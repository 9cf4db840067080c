"""Deterministic packing of GRPO responses into physical learner micro-batches
(``dsv41_train/rl/learner_batch_planner.py:9-85``: same cell syntax, bounds and tie-breaking, so a
plan qualified for one deployment reproduces exactly).

A shape cell ``B:T`` is a measured (batch, input tokens) ceiling. ``plan_learner_microbatches``
covers every response exactly once: without cells, fixed-size batches in index order; with cells,
responses sorted by (length, index) are taken greedily into the cell that fits the most of them
(ties: tighter token bound, then the smaller batch). ``plan_response_ownership`` deals the 8
batches of a G32 group round-robin over ranks, padding with zero-loss placeholders so every rank
runs the same number of collectives.
"""

from __future__ import annotations

MAX_B, MAX_T = 32, 2047


def parse_learner_batch_shapes(text):
    if text is None:
        return None
    if not isinstance(text, str) or not text:
        raise ValueError("learner batch shapes require comma-separated integer B:T cells")
    cells = []
    for item in text.split(","):
        parts = item.split(":")
        if len(parts) != 2 or any(not p.isascii() or not p.isdecimal() for p in parts):
            raise ValueError("learner batch shapes require comma-separated integer B:T cells")
        b, t = map(int, parts)
        if not 1 <= b <= MAX_B or not 1 <= t <= MAX_T:
            raise ValueError("learner batch shape bounds must be B1..32:T1..2047")
        cell = {"max_batch_size": b, "max_model_input_tokens": t}
        if cell in cells:
            raise ValueError("duplicate learner batch shape cell")
        cells.append(cell)
    return sorted(cells, key=lambda c: (c["max_batch_size"], c["max_model_input_tokens"]))


def _valid_cells(shapes) -> bool:
    return bool(shapes) and all(
        set(c) == {"max_batch_size", "max_model_input_tokens"} and type(c["max_batch_size"]) is int
        and 1 <= c["max_batch_size"] <= MAX_B and type(c["max_model_input_tokens"]) is int
        and 1 <= c["max_model_input_tokens"] <= MAX_T for c in shapes)


def plan_learner_microbatches(input_lengths, fixed_size, shapes=None):
    if (type(fixed_size) is not int or not 1 <= fixed_size <= MAX_B or not input_lengths
            or any(type(n) is not int or not 1 <= n <= MAX_T for n in input_lengths)):
        raise ValueError("learner planner requires physical B1..32 and nonempty input lengths1..2047")
    n = len(input_lengths)
    if shapes is None:
        return [{"response_indices": list(range(s, min(s + fixed_size, n))), "qualified_shape_cell": None}
                for s in range(0, n, fixed_size)]
    if not _valid_cells(shapes):
        raise ValueError("learner planner requires explicit qualified B:T cells")
    if any(all(length > c["max_model_input_tokens"] for c in shapes) for length in input_lengths):
        raise ValueError("qualified learner batch shapes do not cover every actual response length")
    order = sorted(range(n), key=lambda i: (input_lengths[i], i))
    plan, cursor = [], 0
    while cursor < n:
        best = None
        for cell in shapes:
            fit = 0
            while (fit < cell["max_batch_size"] and cursor + fit < n
                   and input_lengths[order[cursor + fit]] <= cell["max_model_input_tokens"]):
                fit += 1
            if fit:
                key = (-fit, cell["max_model_input_tokens"], cell["max_batch_size"])
                if best is None or key < best[0]:
                    best = (key, fit, cell)
        _, fit, cell = best
        plan.append({"response_indices": order[cursor:cursor + fit], "qualified_shape_cell": dict(cell)})
        cursor += fit
    return plan


def plan_response_ownership(input_lengths, rank, world_size):
    batches = plan_learner_microbatches(input_lengths, 4)
    if len(input_lengths) != 32:
        raise ValueError("response ownership requires the complete G32 group")
    if type(world_size) is not int or not 1 <= world_size <= 32 or type(rank) is not int or not 0 <= rank < world_size:
        raise ValueError("response ownership requires rank within world size 1..32")
    slots = -(-len(batches) // world_size) * world_size
    return [dict(batches[i if i < len(batches) else 0], is_placeholder=i >= len(batches))
            for i in range(rank, slots, world_size)]


__all__ = ["parse_learner_batch_shapes", "plan_learner_microbatches", "plan_response_ownership"]
