"""Leo configurations used by the tests and the benchmark.

Field names and defaults follow ``crates/leo-core/src/config.rs:8-156``; the
base values are ``configs/probe.toml`` of the reference.  The numbered
configurations restate the benchmark table (probe-sized CPU case, 65,536-unit
single GPU, 262,144-unit Zipf single GPU, 128 workers over several GPUs):

* ``baseline1``: probe.toml with ``synapses_per_neuron = 32``,
  ``input_fanout = 32``, ``eligibility_decay = 0.9``; 4 workers, 64 stories of
  256-1024 bytes, story seed 0.
* ``baseline2``: N = 65,536 (128 blocks x 512), S = 64, F = 64, keep 8,
  ``max_active_global = 1024``, ``target_activity = 0.01``, trace decay 0.9,
  32 workers, stories of 256-1024 bytes.
* ``baseline3``: N = 262,144 (256 blocks x 1024), S = 128 with Zipf(1.1)
  target skew, keep 4, ``max_active_global = 1024``,
  ``target_activity = 0.0039``, 64 workers, stories of 512-2048 bytes.
* ``baseline4``: ``baseline3`` with 128 workers sharded across GPUs.

Every synthetic configuration uses fan-out synapse lists with uniformly drawn
(or Zipf-drawn) targets and weights ``|N(0, 1/sqrt(S))|`` signed by source
type, because the reference's sign rules (``model.rs:362-379``) forbid
negative excitatory weights.  The input projection, output projection,
thresholds and neuron types come from the reference initializer
(``model.rs:79-158``).
"""

from __future__ import annotations

import ctypes as C
import tomllib
from dataclasses import asdict, dataclass, fields, replace

import numpy as np

from .ctypes_types import (
    LeoB200Config,
    TOPOLOGY_REFERENCE,
    TOPOLOGY_UNIFORM,
    TOPOLOGY_ZIPF,
)


@dataclass(frozen=True)
class Config:
    # [model]
    name: str = "Leo-probe"
    seed: int = 1337
    neuron_count: int = 4096
    block_count: int = 128
    neurons_per_block: int = 32
    branches_per_neuron: int = 4
    excitatory_fraction: float = 0.8
    synapses_per_neuron: int = 16
    input_fanout: int = 32
    max_active_per_block: int = 2
    max_active_global: int = 192
    # [dynamics]
    branch_decay: float = 0.85
    membrane_decay: float = 0.90
    fatigue_decay: float = 0.97
    fatigue_gain: float = 0.02
    refractory_ticks: int = 1
    target_activity: float = 0.01
    threshold_homeostasis_rate: float = 0.0001
    population_inhibition_rate: float = 0.05
    population_inhibition_max: float = 2.0
    adaptation_fast_decay: float = 0.95
    adaptation_medium_decay: float = 0.99
    adaptation_slow_decay: float = 0.999
    adaptation_fast_gain: float = 0.005
    adaptation_medium_gain: float = 0.001
    adaptation_slow_gain: float = 0.0002
    membrane_reset_fraction: float = 0.10
    # [learning]
    output_learning_rate: float = 0.002
    recurrent_learning_rate: float = 0.0005
    inhibitory_learning_rate: float = 0.00002
    eligibility_decay: float = 0.95
    eligibility_epsilon: float = 0.00001
    surrogate_width: float = 0.25
    surrogate_gain: float = 0.10
    max_update: float = 0.01
    weight_min: float = -1.0
    weight_max: float = 1.0
    provisional_strength: float = 0.20
    training_strength: float = 1.0
    verified_strength: float = 1.0
    plasticity_window: int = 1
    end_document_weight: float = 4.0
    # [context]
    context_embedding_dim: int = 16
    context_max_order: int = 6
    context_slots_per_order: int = 4096
    context_probe_limit: int = 4
    context_learning_rate: float = 0.02
    context_confidence_observations: int = 8
    context_dropout_rate: float = 0.5
    # [replay]
    replay_fraction: float = 0.30
    replay_segment_bytes: int = 32
    replay_stateful_batch: bool = False
    replay_teaching_replays: int = 1
    replay_max_verified_replays: int = 4
    # [training]: run-loop limits; stored in checkpoints, unused by the story step
    training_max_dataset_passes: int = 3
    training_validate_every_bytes: int = 500_000
    training_checkpoint_every_bytes: int = 500_000
    training_early_stop_checks: int = 3
    training_minimum_relative_improvement: float = 0.005

    def to_c(self) -> LeoB200Config:
        c = LeoB200Config()
        a = c.abi
        d = asdict(self)
        for name, _ in a._fields_:
            setattr(a, name, d[name])
        h = c.host
        h.seed = self.seed
        h.excitatory_fraction = self.excitatory_fraction
        h.provisional_strength = self.provisional_strength
        h.training_strength = self.training_strength
        h.verified_strength = self.verified_strength
        h.plasticity_window = self.plasticity_window
        h.end_document_weight = self.end_document_weight
        h.context_dropout_rate = self.context_dropout_rate
        h.replay_fraction = self.replay_fraction
        h.replay_segment_bytes = self.replay_segment_bytes
        return c

    @property
    def context_slots(self) -> int:
        return self.context_max_order * self.context_slots_per_order



# ---------------------------------------------------------------- TOML text (config.rs:242-249, 521-523)

class ConfigurationError(ValueError):
    """An invalid configuration (LeoError::configuration, crates/leo-core/src/lib.rs)."""


# Tables and keys in the declaration order of the reference structs
# (config.rs:10-156); each key maps to the Config attribute ``prefix + key``.
TOML_TABLES = (
    ("model", "", ("name", "seed", "neuron_count", "block_count", "neurons_per_block", "branches_per_neuron",
                   "excitatory_fraction", "synapses_per_neuron", "input_fanout", "max_active_per_block",
                   "max_active_global")),
    ("dynamics", "", ("branch_decay", "membrane_decay", "fatigue_decay", "fatigue_gain", "refractory_ticks",
                      "target_activity", "threshold_homeostasis_rate", "population_inhibition_rate",
                      "population_inhibition_max", "adaptation_fast_decay", "adaptation_medium_decay",
                      "adaptation_slow_decay", "adaptation_fast_gain", "adaptation_medium_gain",
                      "adaptation_slow_gain", "membrane_reset_fraction")),
    ("learning", "", ("output_learning_rate", "recurrent_learning_rate", "inhibitory_learning_rate",
                      "eligibility_decay", "eligibility_epsilon", "surrogate_width", "surrogate_gain", "max_update",
                      "weight_min", "weight_max", "provisional_strength", "training_strength", "verified_strength",
                      "plasticity_window", "end_document_weight")),
    ("context", "context_", ("max_order", "embedding_dim", "slots_per_order", "probe_limit", "learning_rate",
                             "confidence_observations", "dropout_rate")),
    ("replay", "replay_", ("fraction", "segment_bytes", "stateful_batch", "teaching_replays",
                           "max_verified_replays")),
    ("training", "training_", ("max_dataset_passes", "validate_every_bytes", "checkpoint_every_bytes",
                               "early_stop_checks", "minimum_relative_improvement")),
)
# Keys the reference deserializer fills in when absent (config.rs:93-94, 121-122).
TOML_DEFAULTS = {("learning", "plasticity_window"): 1, ("replay", "stateful_batch"): False}
# Integer fields declared u32 in the reference; every other integer is u64/usize.
_U32_FIELDS = {"context_confidence_observations"}


def _field_kind(attr: str) -> type:
    return {f.name: f.type for f in fields(Config)}[attr]


def _f32_text(value: float) -> str:
    """Shortest decimal that reads back as the same f32, always with a point."""
    return np.format_float_positional(np.float32(value), unique=True, trim="0")


def _f32_canonical(value: float) -> float:
    return float(_f32_text(value))


def _toml_string(text: str) -> str:
    out = ['"']
    for ch in text:
        code = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif ch == "\n":
            out.append("\\n")
        elif ch == "\t":
            out.append("\\t")
        elif ch == "\r":
            out.append("\\r")
        elif code < 0x20 or code == 0x7F:
            out.append(f"\\u{code:04X}")
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def config_to_toml(config: Config) -> str:
    """TOML text of a configuration: the six tables in declaration order.

    Floats are written as the shortest decimal of their f32 value, so the text
    reads back to a bit-identical configuration.  The reference renders this
    text with the ``toml`` crate 0.8.19 (``to_string_pretty``); its float and
    string spellings are not pinned here, and only the parsed values have to
    agree.
    """
    lines: list[str] = []
    for table, prefix, keys in TOML_TABLES:
        if lines:
            lines.append("")
        lines.append(f"[{table}]")
        for key in keys:
            value = getattr(config, prefix + key)
            kind = _field_kind(prefix + key)
            if kind in ("str", str):
                text = _toml_string(value)
            elif kind in ("bool", bool):
                text = "true" if value else "false"
            elif kind in ("float", float):
                text = _f32_text(value)
            else:
                text = str(int(value))
            lines.append(f"{key} = {text}")
    return "\n".join(lines) + "\n"


def config_from_toml(text: str) -> Config:
    """Config::from_toml (config.rs:242-249): unknown tables or keys, missing
    keys without a default, and values of the wrong type are errors; the result
    is validated."""
    try:
        doc = tomllib.loads(text)
    except tomllib.TOMLDecodeError as e:
        raise ConfigurationError(f"invalid TOML configuration: {e}") from None
    tables = {t for t, _, _ in TOML_TABLES}
    unknown = set(doc) - tables
    if unknown:
        raise ConfigurationError(f"invalid TOML configuration: unknown field {sorted(unknown)[0]!r}")
    kwargs: dict = {}
    for table, prefix, keys in TOML_TABLES:
        body = doc.get(table)
        if not isinstance(body, dict):
            raise ConfigurationError(f"invalid TOML configuration: missing field {table!r}")
        extra = set(body) - set(keys)
        if extra:
            raise ConfigurationError(f"invalid TOML configuration: unknown field {sorted(extra)[0]!r} in [{table}]")
        for key in keys:
            attr = prefix + key
            if key not in body:
                if (table, key) not in TOML_DEFAULTS:
                    raise ConfigurationError(f"invalid TOML configuration: missing field {key!r} in [{table}]")
                kwargs[attr] = TOML_DEFAULTS[(table, key)]
                continue
            value = body[key]
            kind = _field_kind(attr)
            if kind in ("str", str):
                ok = isinstance(value, str)
            elif kind in ("bool", bool):
                ok = isinstance(value, bool)
            elif kind in ("float", float):
                ok = isinstance(value, (int, float)) and not isinstance(value, bool)
                if ok:
                    with np.errstate(over="ignore"):
                        value = _f32_canonical(value)
            else:
                limit = 2**32 if attr in _U32_FIELDS else 2**64
                ok = isinstance(value, int) and not isinstance(value, bool) and 0 <= value < limit
            if not ok:
                raise ConfigurationError(f"invalid TOML configuration: invalid value for {key!r} in [{table}]")
            kwargs[attr] = value
    config = Config(**kwargs)
    validate_config(config)
    return config


def validate_config(config: Config) -> None:
    """Config::validate (config.rs:251-519): the kernel-facing fields through
    the native validator, then the run-loop fields the kernels never read."""
    from . import native

    c = config.to_c()
    if native.lib().leo_b200_config_validate(C.byref(c)) != 0:
        raise ConfigurationError(native.lib().leo_b200_last_error().decode())
    if not config.name.strip():
        raise ConfigurationError("model.name must not be empty")
    if config.replay_segment_bytes == 0 or config.replay_teaching_replays == 0 \
            or config.replay_max_verified_replays == 0:
        raise ConfigurationError("all replay limits must be positive")
    if config.training_max_dataset_passes == 0 or config.training_validate_every_bytes == 0 \
            or config.training_checkpoint_every_bytes == 0 or config.training_early_stop_checks == 0:
        raise ConfigurationError("all training limits must be positive")
    mri = np.float32(config.training_minimum_relative_improvement)
    if not np.isfinite(mri) or mri < 0:
        raise ConfigurationError("minimum_relative_improvement must be finite and nonnegative")


@dataclass(frozen=True)
class Workload:
    """A configuration plus the synthetic story stream that exercises it."""

    name: str
    config: Config
    topology: int
    workers: int
    stories: int
    min_story_bytes: int
    max_story_bytes: int
    story_seed: int = 0


PROBE = Config()

TEST = Config(
    name="Leo-test", replay_max_verified_replays=2, training_max_dataset_passes=2,
    training_validate_every_bytes=512, training_checkpoint_every_bytes=1024,
    neuron_count=128, block_count=8, neurons_per_block=16, synapses_per_neuron=8, input_fanout=8,
    max_active_per_block=2, max_active_global=8, target_activity=0.04, inhibitory_learning_rate=0.00005,
    context_embedding_dim=8, context_max_order=4, context_slots_per_order=128, context_learning_rate=0.08,
    context_confidence_observations=2, context_dropout_rate=0.0, replay_segment_bytes=8,
)

BASELINE1 = replace(PROBE, synapses_per_neuron=32, input_fanout=32, eligibility_decay=0.9)

BASELINE2 = replace(
    PROBE, neuron_count=65536, block_count=128, neurons_per_block=512, synapses_per_neuron=64, input_fanout=64,
    max_active_per_block=8, max_active_global=1024, target_activity=0.01, eligibility_decay=0.9,
)

BASELINE3 = replace(
    PROBE, neuron_count=262144, block_count=256, neurons_per_block=1024, synapses_per_neuron=128,
    input_fanout=64, max_active_per_block=4, max_active_global=1024, target_activity=0.0039,
)

WORKLOADS = {
    "test": Workload("test", TEST, TOPOLOGY_REFERENCE, 4, 16, 8, 48),
    "probe": Workload("probe", PROBE, TOPOLOGY_REFERENCE, 4, 64, 256, 1024),
    "baseline1": Workload("baseline1", BASELINE1, TOPOLOGY_UNIFORM, 4, 64, 256, 1024),
    "baseline2": Workload("baseline2", BASELINE2, TOPOLOGY_UNIFORM, 32, 10_000, 256, 1024),
    "baseline2-replay-off": Workload("baseline2-replay-off", replace(BASELINE2, replay_fraction=0.0),
                                     TOPOLOGY_UNIFORM, 32, 10_000, 256, 1024),
    # Small case of the baseline2 model for kernel captures: 2 lanes of short stories.
    "profile": Workload("profile", BASELINE2, TOPOLOGY_UNIFORM, 2, 64, 80, 96),
    "baseline3": Workload("baseline3", BASELINE3, TOPOLOGY_ZIPF, 64, 50_000, 512, 2048),
    # Small case of the baseline3 model: 4 lanes of short stories.
    "baseline3-small": Workload("baseline3-small", BASELINE3, TOPOLOGY_ZIPF, 4, 64, 64, 128),
    # Small case of the baseline3 model for kernel captures: 2 lanes of short stories.
    "baseline3-profile": Workload("baseline3-profile", BASELINE3, TOPOLOGY_ZIPF, 2, 64, 80, 96),
    "baseline4": Workload("baseline4", BASELINE3, TOPOLOGY_ZIPF, 128, 50_000, 512, 2048),
}


def c_config(config: Config) -> LeoB200Config:
    return config.to_c()


__all__ = ["Config", "ConfigurationError", "config_from_toml", "config_to_toml", "validate_config", "Workload", "WORKLOADS", "PROBE", "TEST", "BASELINE1", "BASELINE2", "BASELINE3", "c_config"]
_ = C  # re-exported types keep ctypes imported for callers
