"""Host-side persistent model (crates/leo-core/src/model.rs:65-76) as numpy
arrays, exchanged with the C ABI through ``LeoB200HostModel`` views."""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import native
from .configs import Config
from .ctypes_types import LeoB200HostModel, LeoB200Statistics, OUTPUT_CLASSES, SYMBOL_COUNT

DTYPES = {
    "threshold": np.float32, "excitability": np.float32, "neuron_type": np.uint8,
    "recurrent_target": np.uint32, "recurrent_branch": np.uint8, "recurrent_delay": np.uint8,
    "recurrent_weight": np.float32, "input_target": np.uint32, "input_branch": np.uint8,
    "input_weight": np.float32, "output_weight": np.float32, "output_bias": np.float32,
    "context_keys": np.uint64, "context_embeddings": np.float32, "context_observations": np.uint32,
    "context_output_weight": np.float32,
}


def array_sizes(cfg: Config) -> dict[str, int]:
    n, s, f, d = cfg.neuron_count, cfg.synapses_per_neuron, cfg.input_fanout, cfg.context_embedding_dim
    ctx = cfg.context_slots
    return {
        "threshold": n, "excitability": n, "neuron_type": n,
        "recurrent_target": n * s, "recurrent_branch": n * s, "recurrent_delay": n * s, "recurrent_weight": n * s,
        "input_target": SYMBOL_COUNT * f, "input_branch": SYMBOL_COUNT * f, "input_weight": SYMBOL_COUNT * f,
        "output_weight": OUTPUT_CLASSES * n, "output_bias": OUTPUT_CLASSES,
        "context_keys": ctx, "context_embeddings": ctx * d, "context_observations": ctx,
        "context_output_weight": OUTPUT_CLASSES * d,
    }


class HostModel:
    """A model whose tensors are numpy arrays in the checkpoint layout."""

    def __init__(self, config: Config, arrays: dict[str, np.ndarray] | None = None):
        self.config = config
        sizes = array_sizes(config)
        if arrays is None:
            arrays = {k: np.zeros(v, dtype=DTYPES[k]) for k, v in sizes.items()}
        self.arrays = {k: np.ascontiguousarray(arrays[k], dtype=DTYPES[k]) for k in DTYPES}
        for k, v in sizes.items():
            if self.arrays[k].size != v:
                raise ValueError(f"{k}: expected {v} elements, got {self.arrays[k].size}")
        self.generation = 0
        self.parameter_revision = 0
        self.statistics = LeoB200Statistics()

    def view(self) -> LeoB200HostModel:
        hm = LeoB200HostModel()
        hm.config = self.config.to_c()
        hm.generation = self.generation
        hm.parameter_revision = self.parameter_revision
        hm.statistics = self.statistics
        for name, a in self.arrays.items():
            setattr(hm, name, a.ctypes.data_as(type(getattr(hm, name))))
        return hm

    def absorb_scalars(self, hm: LeoB200HostModel) -> None:
        self.generation = hm.generation
        self.parameter_revision = hm.parameter_revision
        self.statistics = hm.statistics

    @classmethod
    def initialize(cls, config: Config, topology: int) -> "HostModel":
        """Model::initialize (model.rs:79-158) with the chosen topology."""
        m = cls(config)
        hm = m.view()
        native.check(native.lib().leo_b200_model_initialize(C.byref(hm.config), topology, C.byref(hm)))
        m.absorb_scalars(hm)
        return m

    def validate(self) -> None:
        hm = self.view()
        native.check(native.lib().leo_b200_model_validate(C.byref(hm)))

    def training_state_hash(self) -> bytes:
        hm = self.view()
        out = (C.c_uint8 * 32)()
        native.check(native.lib().leo_b200_training_state_hash(C.byref(hm), out))
        return bytes(out)

    def copy(self) -> "HostModel":
        m = HostModel(self.config, {k: v.copy() for k, v in self.arrays.items()})
        m.generation = self.generation
        m.parameter_revision = self.parameter_revision
        stats = LeoB200Statistics()
        C.memmove(C.byref(stats), C.byref(self.statistics), C.sizeof(stats))
        m.statistics = stats
        return m
