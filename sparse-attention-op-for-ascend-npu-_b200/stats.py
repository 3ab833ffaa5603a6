"""Process-wide counters for TriangleMix routing and launches.

The method names and the exported counter names follow the reference
plugin's runtime statistics (package/src/vllm_ascend_trianglemix/stats.py:14-514
in the reference project), so dashboards and tests built on the snapshot keep
working:

* planner counters are recorded once per plan (a plan is shared by every
  selected layer of a step): ``request_total``, ``request_planner_eligible``,
  ``request_planner_ineligible``, ``routing_ns`` and the per-reason
  ``fallback_reasons``;
* layer counters are recorded per selected layer call: ``layer_direct`` (this
  library's kernel ran), ``layer_fia`` (the stock backend ran; the reference's
  name for its fallback path) with ``layer_fia_reason:<reason>``,
  ``single_launch``, ``estimated_saved_qk`` and the host enqueue time;
* ``performance`` derives rates from them (planner eligibility, routing and
  host enqueue time per request / launch);
* ``recent`` keeps the last ``recent_capacity`` plans with their requests and
  what the layers actually did with them.

All updates take one lock; the hot path records one small dict update per
layer call.
"""

from __future__ import annotations

import threading
from collections import Counter, OrderedDict
from copy import deepcopy
from typing import Any

from .planning import FallbackReason, TriangleBatchPlan


def _empty_execution() -> dict[str, Any]:
    return {"observed_route": "unobserved", "layer_direct": 0, "layer_fia": 0,
            "layer_hit_rate": 0.0, "fallback_reasons": {}, "single_launch": 0,
            "estimated_saved_qk": 0, "host_enqueue_ns_total": 0, "host_enqueue_ns_max": 0,
            "timing_scope": "host_enqueue_not_device_latency"}


class TriangleMixRuntimeStats:
    _SEEN_CAPACITY = 8192

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._reset_locked()
        self._recent_capacity = 256
        self._log_interval = 0

    def _reset_locked(self) -> None:
        self._counters: Counter[str] = Counter()
        self._reasons: Counter[str] = Counter()
        self._layer_direct: Counter[str] = Counter()
        self._layer_fia: Counter[str] = Counter()
        self._seen: OrderedDict[int, None] = OrderedDict()
        self._recent: OrderedDict[int, dict[str, Any]] = OrderedDict()
        self._next_log = 0

    def configure(self, recent_capacity: int, log_interval: int = 0) -> None:
        if recent_capacity < 0 or log_interval < 0:
            raise ValueError("TriangleMix stats configuration must be non-negative")
        with self._lock:
            self._recent_capacity = recent_capacity
            while len(self._recent) > recent_capacity:
                self._recent.popitem(last=False)
            self._log_interval = log_interval
            total = self._counters["request_total"]
            self._next_log = (total // log_interval + 1) * log_interval if log_interval else 0

    # ------------------------------------------------------------ planner
    def record_planner_decision(self, plan: TriangleBatchPlan) -> None:
        """Record a plan's request-level decisions once, however many layers use it."""
        with self._lock:
            if plan.plan_id in self._seen:
                return
            self._seen[plan.plan_id] = None
            if len(self._seen) > self._SEEN_CAPACITY:
                self._seen.popitem(last=False)
            requests = plan.requests[:plan.batch_size]
            eligible = sum(1 for r in requests if r.eligible)
            self._counters["routing_ns"] += plan.routing_ns
            self._counters["request_total"] += plan.batch_size
            self._counters["request_planner_eligible"] += eligible
            self._counters["request_planner_ineligible"] += plan.batch_size - eligible
            for r in requests:
                if not r.eligible:
                    self._reasons[r.reason.value] += 1
            if self._recent_capacity:
                self._recent[plan.plan_id] = {
                    "plan_id": plan.plan_id, "state": plan.state_name,
                    "batch_size": plan.batch_size,
                    "route": "planner_eligible" if plan.direct else "planner_ineligible",
                    "reason": plan.primary_reason.value, "execution": _empty_execution(),
                    "requests": [{"slot": r.request_index, "q_begin": r.q_begin,
                                  "q_end": r.q_end, "seq_len": r.seq_len,
                                  "prompt_len": r.prompt_len, "saved_qk": r.saved_qk,
                                  "eligible": r.eligible, "reason": r.reason.value}
                                 for r in requests]}
                while len(self._recent) > self._recent_capacity:
                    self._recent.popitem(last=False)

    def record_request_decision(self, plan: TriangleBatchPlan, *, direct: bool | None = None,
                                reason: FallbackReason | None = None) -> None:
        """Older name of record_planner_decision (the extra arguments are ignored)."""
        del direct, reason
        self.record_planner_decision(plan)

    # ------------------------------------------------------------ layers
    def _execution_locked(self, plan_id: int | None) -> dict[str, Any] | None:
        entry = self._recent.get(plan_id) if plan_id is not None else None
        return entry["execution"] if entry is not None else None

    @staticmethod
    def _observe(execution: dict[str, Any]) -> None:
        direct, fia = execution["layer_direct"], execution["layer_fia"]
        execution["layer_hit_rate"] = direct / (direct + fia) if direct + fia else 0.0
        execution["observed_route"] = ("mixed" if direct and fia else
                                       "all_direct" if direct else "all_fia")

    def record_layer_dispatch(self, *, plan_id: int, layer_index: int | None, saved_qk: int,
                              host_enqueue_ns: int, request_index: int = 0,
                              launches: int = 1) -> None:
        """A selected layer ran this library's kernel (``launches`` launches)."""
        del request_index
        with self._lock:
            c = self._counters
            c["layer_direct"] += 1
            c["single_launch"] += launches
            c["estimated_saved_qk"] += saved_qk
            c["host_enqueue_ns"] += host_enqueue_ns
            c["host_enqueue_ns_max"] = max(c["host_enqueue_ns_max"], host_enqueue_ns)
            self._layer_direct[str(layer_index)] += 1
            ex = self._execution_locked(plan_id)
            if ex is not None:
                ex["layer_direct"] += 1
                ex["single_launch"] += launches
                ex["estimated_saved_qk"] += saved_qk
                ex["host_enqueue_ns_total"] += host_enqueue_ns
                ex["host_enqueue_ns_max"] = max(ex["host_enqueue_ns_max"], host_enqueue_ns)
                self._observe(ex)

    def record_layer_fallback(self, *, plan_id: int | None = None, layer_index: int | None,
                              reason: FallbackReason,
                              request_indices: tuple[int, ...] = ()) -> None:
        """A selected layer stayed on the stock attention backend."""
        del request_indices
        with self._lock:
            self._counters["layer_fia"] += 1
            self._counters[f"layer_fia_reason:{reason.value}"] += 1
            self._layer_fia[str(layer_index)] += 1
            ex = self._execution_locked(plan_id)
            if ex is not None:
                ex["layer_fia"] += 1
                reasons = ex["fallback_reasons"]
                reasons[reason.value] = reasons.get(reason.value, 0) + 1
                self._observe(ex)

    def record_runtime_error(self, *, stage: str) -> None:
        with self._lock:
            self._counters["runtime_error"] += 1
            self._counters[f"runtime_error:{stage}"] += 1

    # ------------------------------------------------------------ export
    def _snapshot_locked(self) -> dict[str, Any]:
        c = self._counters
        requests, direct = c["request_total"], c["layer_direct"]
        return {
            "counters": dict(c),
            "fallback_reasons": dict(self._reasons),
            "layers": {"direct": dict(self._layer_direct), "fia": dict(self._layer_fia)},
            "performance": {
                "planner_eligibility_rate": (c["request_planner_eligible"] / requests
                                             if requests else 0.0),
                "routing_us_per_request": c["routing_ns"] / requests / 1e3 if requests else 0.0,
                "host_enqueue_us_per_launch": (c["host_enqueue_ns"] / direct / 1e3
                                               if direct else 0.0),
                "host_enqueue_us_max": c["host_enqueue_ns_max"] / 1e3,
                "host_enqueue_timing_scope": "host_wall_time_not_device_latency",
            },
            "recent": deepcopy(list(self._recent.values())),
        }

    def snapshot(self, reset: bool = False) -> dict[str, Any]:
        with self._lock:
            snap = self._snapshot_locked()
            if reset:
                capacity, interval = self._recent_capacity, self._log_interval
                self._reset_locked()
                self._recent_capacity, self._log_interval = capacity, interval
                self._next_log = interval
            return snap

    def structured_log_if_due(self) -> dict[str, Any] | None:
        """A snapshot each time request_total crosses a multiple of the log interval."""
        with self._lock:
            if not self._log_interval or self._counters["request_total"] < self._next_log:
                return None
            total = self._counters["request_total"]
            self._next_log = (total // self._log_interval + 1) * self._log_interval
            return {"event": "trianglemix_stats", **self._snapshot_locked()}


_STATS = TriangleMixRuntimeStats()


def stats_snapshot(reset: bool = False) -> dict[str, Any]:
    return _STATS.snapshot(reset=reset)


def runtime_stats() -> TriangleMixRuntimeStats:
    return _STATS
