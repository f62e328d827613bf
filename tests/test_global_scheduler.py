"""Cross-engine token budgets and preemption-donor selection."""
from kapsl_sdk_b200.llm.global_scheduler import GlobalKvScheduler, PreemptionRequest


def test_budgets_weights_cap_idle_and_rounding():
    g = GlobalKvScheduler(1000)
    g.register(1, 1)
    g.register(2, 2)
    g.register(3, 1)
    # none active -> all active: 250 / 500 / 250 (cap 900)
    assert g.allocate_budgets() == {1: 250, 2: 500, 3: 250}
    g.set_active(2, True)
    # only engine 2 active: its share 500 + idle 250 + 250 (idle may exceed the cap)
    assert g.allocate_budgets() == {1: 0, 2: 1000, 3: 0}
    g.set_active(1, True)
    assert g.allocate_budgets() == {1: 500, 2: 500, 3: 0}
    h = GlobalKvScheduler(100)
    for e in (1, 2, 3):
        h.register(e, 1)
    assert h.allocate_budgets() == {1: 34, 2: 33, 3: 33}  # rounding remainder to the first engine
    solo = GlobalKvScheduler(1000)
    solo.register(7, 5)
    assert solo.budget_for(7) == 900  # single engine capped at 90%
    g.deregister(2)
    assert g.engine_count == 2


def test_preemption_donor():
    g = GlobalKvScheduler(100)
    for e in (1, 2, 3, 4):
        g.register(e)
    req = PreemptionRequest(requesting_engine_id=1, blocks_needed=10, request_priority=5)
    prios = {1: 9, 2: 3, 3: 1, 4: 1}
    free = {2: 50, 3: 5, 4: 20}
    assert g.find_preemption_donor(req, prios, free) == 4  # 3 cannot free enough
    assert g.find_preemption_donor(PreemptionRequest(1, 100, 5), prios, free) is None
