"""AutoScaler: replica-count decisions with hysteresis
(crates/kapsl-core/src/auto_scaler.rs:5-291).

Scale up by one when the average queue depth per replica stays above the
policy target for 20 s (up to ``max_replicas`` and the replicas the queue
needs); scale down by one when the total queue depth stays at or below the
threshold for a cooldown and no scale-up happened within it.  No decision is
taken while metrics are missing or any replica is unhealthy.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Optional

SCALE_UP_HYSTERESIS_S = 20.0
MAX_SCALE_UP_STEP = 1


@dataclass
class ScalingPolicy:
    min_replicas: int = 1
    max_replicas: int = 4
    target_queue_depth: int = 5
    scale_down_threshold: int = 2
    cooldown_seconds: float = 300.0

    def validate(self) -> None:
        if self.min_replicas < 1:
            raise ValueError("min_replicas must be at least 1")
        if self.max_replicas < self.min_replicas:
            raise ValueError("max_replicas must be greater than or equal to min_replicas")
        if self.target_queue_depth == 0:
            raise ValueError("target_queue_depth must be greater than 0")
        if self.cooldown_seconds <= 0:
            raise ValueError("cooldown_seconds must be greater than 0")


@dataclass
class _State:
    last_up: Optional[float] = None
    last_down: Optional[float] = None
    high: float = 0.0
    low: float = 0.0


class AutoScaler:
    def __init__(self, clock=time.monotonic):
        self.policies: dict = {}
        self.states: dict = {}
        self.clock = clock

    def register_policy(self, model_id: int, policy: ScalingPolicy) -> None:
        policy.validate()
        self.policies[model_id] = policy
        self.states[model_id] = _State()

    def get_policy(self, model_id: int) -> ScalingPolicy:
        return self.policies.get(model_id, ScalingPolicy())

    def should_scale_up(self, model_id, current, healthy, queue_depth, elapsed_s, metrics_available=True):
        p = self.get_policy(model_id)
        st = self.states.setdefault(model_id, _State())
        if p.target_queue_depth == 0:
            return None
        if not metrics_available or current == 0 or healthy < current or current >= p.max_replicas:
            st.high = 0.0
            return None
        if queue_depth / current > p.target_queue_depth:
            st.high += elapsed_s
            st.low = 0.0
            if st.high < SCALE_UP_HYSTERESIS_S:
                return None
            needed = min((queue_depth + p.target_queue_depth - 1) // p.target_queue_depth, p.max_replicas)
            if needed > current:
                target = min(current + MAX_SCALE_UP_STEP, needed, p.max_replicas)
                if target > current:
                    st.last_up = self.clock()
                    st.high = 0.0
                    return target
        else:
            st.high = 0.0
        return None

    def should_scale_down(self, model_id, current, healthy, queue_depth, elapsed_s, metrics_available=True):
        p = self.get_policy(model_id)
        st = self.states.setdefault(model_id, _State())
        if not metrics_available or healthy < current:
            st.low = 0.0
            return None
        if current <= p.min_replicas:
            return None
        if queue_depth <= p.scale_down_threshold:
            st.low += elapsed_s
            if st.low >= p.cooldown_seconds:
                now = self.clock()
                can = st.last_down is None or now - st.last_down >= p.cooldown_seconds
                recent_up = st.last_up is not None and now - st.last_up < p.cooldown_seconds
                if can and not recent_up:
                    st.last_down = now
                    st.low = 0.0
                    return max(current - 1, p.min_replicas)
        else:
            st.low = 0.0
        return None

    @staticmethod
    def next_replica_id(existing: list) -> int:
        return max(existing) + 1 if existing else 1
