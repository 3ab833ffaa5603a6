"""Typed TriangleMix plugin configuration (vLLM ``additional_config`` or environment).

Same keys, environment variable names, defaults and validation errors as the
reference plugin's configuration (package/src/vllm_ascend_trianglemix/
config.py:11-197 in the reference project), so a deployment switches over
without touching its configuration.  The section is
``additional_config["trianglemix"]`` (or the top-level ``additional_config``
mapping); a key present there wins over its environment variable.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Mapping

from .kernel import TriangleMixConfig, parse_layer_indices

_TRUE = frozenset({"1", "true", "yes", "on"})
_FALSE = frozenset({"0", "false", "no", "off"})


def coerce_bool(value: object, *, name: str) -> bool:
    """bool, 0/1, or one of the usual true/false words (config.py:16-29)."""
    if isinstance(value, bool):
        return value
    if isinstance(value, int) and value in (0, 1):
        return bool(value)
    if isinstance(value, str):
        word = value.strip().lower()
        if word in _TRUE:
            return True
        if word in _FALSE:
            return False
    raise ValueError(f"TriangleMix {name} must be a boolean, got {value!r}")


# Direct-route thresholds (planner gates, reference kernel.py:240-269) per
# device.  "910b" holds the reference's values, calibrated on Ascend 910B3.
# "b200" comes from the BASELINE config 1 sweep on one B200 (bench.py
# --crossover, arms in alternating order): every chunk with sparse rows (181
# to 2048 of them, 127 K to 13.6 M skipped QK pairs per head) ran 2.2x to
# 21.7x faster through this library than FlashInfer's paged prefill over the
# same 128-token pages, also by the robust bound min(dense) / max(sparse).
# Against this kernel's own all-dense mode the only chunk without a gain is
# the 309-row last chunk of a 2869-token prompt (181 sparse rows, 1.00x), so
# no saved-pairs minimum is kept; chunks below 128 sparse rows were not
# measured and keep the reference's floor.
THRESHOLD_PROFILES: dict[str, dict[str, int]] = {
    "910b": {"min_seq_len": 0, "min_sparse_rows": 128, "min_saved_qk": 913_152,
             "split_min_sparse_rows": 192, "split_min_saved_qk": 1_299_264},
    "b200": {"min_seq_len": 0, "min_sparse_rows": 128, "min_saved_qk": 0,
             "split_min_sparse_rows": 128, "split_min_saved_qk": 0},
}
_THRESHOLD_KEYS = tuple(THRESHOLD_PROFILES["910b"])

# key -> (environment variable, default).  The threshold keys' defaults come
# from the selected profile (threshold_profile, not a key of the reference
# plugin); a threshold key set in the section or its environment variable
# still wins over the profile.
_KEYS: dict[str, tuple[str, Any]] = {
    "threshold_profile": ("VLLM_ASCEND_TRIANGLE_MIX_THRESHOLD_PROFILE", "b200"),
    "enabled": ("VLLM_ASCEND_ENABLE_TRIANGLE_MIX", False),
    "layers": ("VLLM_ASCEND_TRIANGLE_MIX_LAYERS", ""),
    "sink_tokens": ("VLLM_ASCEND_TRIANGLE_MIX_SINK_TOKENS", 8),
    "local_window": ("VLLM_ASCEND_TRIANGLE_MIX_LOCAL_WINDOW", 512),
    "last_rows": ("VLLM_ASCEND_TRIANGLE_MIX_LAST_ROWS", 128),
    "min_seq_len": ("VLLM_ASCEND_TRIANGLE_MIX_DIRECT_MIN_SEQ_LEN", 0),
    "min_sparse_rows": ("VLLM_ASCEND_TRIANGLE_MIX_DIRECT_MIN_SPARSE_ROWS", 128),
    "min_saved_qk": ("VLLM_ASCEND_TRIANGLE_MIX_DIRECT_MIN_SAVED_QK", 913_152),
    "split_min_sparse_rows": ("VLLM_ASCEND_TRIANGLE_MIX_DIRECT_SPLIT_MIN_SPARSE_ROWS", 192),
    "split_min_saved_qk": ("VLLM_ASCEND_TRIANGLE_MIX_DIRECT_SPLIT_MIN_SAVED_QK", 1_299_264),
    "strict": ("VLLM_ASCEND_TRIANGLE_MIX_STRICT", False),
    "stats_recent_capacity": ("VLLM_ASCEND_TRIANGLE_MIX_STATS_RECENT_CAPACITY", 256),
    "stats_log_interval": ("VLLM_ASCEND_TRIANGLE_MIX_STATS_LOG_INTERVAL", 0),
}


def _lookup(section: Mapping[str, Any], key: str) -> Any:
    env, default = _KEYS[key]
    if key in section:
        return section[key]
    raw = os.getenv(env)
    if raw is None:
        return default
    if isinstance(default, bool):
        return coerce_bool(raw, name=env)
    if isinstance(default, int):
        return int(raw)
    return raw


@dataclass(frozen=True)
class PluginConfig:
    """Process configuration shared by the planner and the attention hook."""

    kernel: TriangleMixConfig
    strict: bool = False
    stats_recent_capacity: int = 256
    stats_log_interval: int = 0

    @property
    def enabled(self) -> bool:
        return self.kernel.enabled and bool(self.kernel.layer_indices)


def resolve_plugin_config(vllm_config: object | None) -> PluginConfig:
    """Resolve the typed configuration, preferring ``additional_config.trianglemix``."""
    additional = getattr(vllm_config, "additional_config", None)
    additional = additional if isinstance(additional, Mapping) else {}
    section = additional.get("trianglemix", additional)
    section = section if isinstance(section, Mapping) else {}
    profile_name = str(_lookup(section, "threshold_profile")).strip().lower()
    if profile_name not in THRESHOLD_PROFILES:
        raise ValueError(f"TriangleMix threshold_profile must be one of "
                         f"{sorted(THRESHOLD_PROFILES)}, got {profile_name!r}")
    profile = THRESHOLD_PROFILES[profile_name]

    def threshold(key: str) -> int:
        env, _ = _KEYS[key]
        if key in section or os.getenv(env) is not None:
            return int(_lookup(section, key))
        return profile[key]

    layers = _lookup(section, "layers")
    if isinstance(layers, (list, tuple, set, frozenset)):
        layers = ",".join(str(x) for x in layers)
    kernel = TriangleMixConfig(
        enabled=coerce_bool(_lookup(section, "enabled"), name="enabled"),
        layer_indices=parse_layer_indices(str(layers)),
        sink_tokens=int(_lookup(section, "sink_tokens")),
        local_window=int(_lookup(section, "local_window")),
        last_rows=int(_lookup(section, "last_rows")),
        direct_min_seq_len=threshold("min_seq_len"),
        direct_min_sparse_rows=threshold("min_sparse_rows"),
        direct_min_saved_qk=threshold("min_saved_qk"),
        direct_split_min_sparse_rows=threshold("split_min_sparse_rows"),
        direct_split_min_saved_qk=threshold("split_min_saved_qk"),
    )
    recent = int(_lookup(section, "stats_recent_capacity"))
    interval = int(_lookup(section, "stats_log_interval"))
    if recent < 0 or interval < 0:
        raise ValueError("TriangleMix stats capacities must be non-negative")
    return PluginConfig(kernel=kernel,
                        strict=coerce_bool(_lookup(section, "strict"), name="strict"),
                        stats_recent_capacity=recent, stats_log_interval=interval)
