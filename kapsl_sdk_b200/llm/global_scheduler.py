"""Cross-engine token budget for several engines sharing one device.

Budgets: every registered engine has a share weight; its natural share is
``global_max_tokens * weight / sum(weights)``.  Active engines get their
share capped at ``max_single_engine_permille / 1000`` of the total; idle
engines get 0 and their shares go (uncapped) to the first active engine in
registration order, which also receives the integer-rounding remainder up to
the cap.  With no engine marked active, all count as active.  Preemption
donor: among the other engines whose priority is below the request's and
that can free enough blocks, the lowest-priority one (first registered on a
tie).  These are the reference's rules (crates/kapsl-llm/src/global_scheduler.rs:1-331),
so mixed deployments split capacity the same way; unlike the reference,
:meth:`apply` pushes the budgets into the engines' per-step token budgets.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional


@dataclass
class _State:
    weight: int
    used: int = 0
    active: bool = False


@dataclass
class PreemptionRequest:
    requesting_engine_id: int
    blocks_needed: int
    request_priority: int


class GlobalKvScheduler:
    def __init__(self, global_max_tokens: int, max_single_engine_permille: int = 900):
        self.global_max_tokens = global_max_tokens
        self.max_single_engine_permille = min(1000, max(100, max_single_engine_permille))
        self._engines: dict[int, _State] = {}
        self._order: list[int] = []

    def register(self, engine_id: int, share_weight: int = 1) -> None:
        if engine_id not in self._engines:
            self._order.append(engine_id)
        self._engines[engine_id] = _State(max(1, share_weight))

    def deregister(self, engine_id: int) -> None:
        self._engines.pop(engine_id, None)
        self._order = [e for e in self._order if e != engine_id]

    def set_active(self, engine_id: int, active: bool) -> None:
        if engine_id in self._engines:
            self._engines[engine_id].active = active

    def report_usage(self, engine_id: int, used_tokens: int) -> None:
        if engine_id in self._engines:
            self._engines[engine_id].used = used_tokens

    @property
    def engine_count(self) -> int:
        return len(self._engines)

    def allocate_budgets(self) -> dict:
        if not self._engines or self.global_max_tokens == 0:
            return {}
        G = self.global_max_tokens
        all_active = not any(s.active for s in self._engines.values())
        total_w = max(1, sum(s.weight for s in self._engines.values()))
        cap = G * self.max_single_engine_permille // 1000
        budgets, idle, natural_sum = {}, 0, 0
        for eid in self._order:
            s = self._engines[eid]
            natural = G * s.weight // total_w
            natural_sum += natural
            if s.active or all_active:
                budgets[eid] = min(natural, cap)
            else:
                budgets[eid] = 0
                idle += natural
        first = next((e for e in self._order if budgets[e] > 0), None)
        if first is not None:
            budgets[first] += idle
            rounding = G - natural_sum
            if rounding > 0:
                budgets[first] += min(rounding, max(0, cap - budgets[first]))
        return budgets

    def budget_for(self, engine_id: int) -> Optional[int]:
        return self.allocate_budgets().get(engine_id)

    def find_preemption_donor(self, req: PreemptionRequest, priorities: dict, freeable_blocks: dict) -> Optional[int]:
        cands = [e for e in self._order if e != req.requesting_engine_id and e in priorities
                 and priorities[e] < req.request_priority and freeable_blocks.get(e, 0) >= req.blocks_needed]
        return min(cands, key=lambda e: priorities[e]) if cands else None

    def apply(self, engines: dict) -> dict:
        """Set each engine's per-step token budget (``engines``: id -> LLMEngine);
        an engine with budget 0 keeps a budget of 1 token so it can still drain."""
        b = self.allocate_budgets()
        for eid, eng in engines.items():
            if eid in b:
                eng.scheduler.max_tokens = max(1, b[eid])
        return b
