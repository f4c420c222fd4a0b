"""Host-side model logic of the product against the oracle, on CPU.

``leo_b200_model_initialize`` restates ``Model::initialize``
(``crates/leo-core/src/model.rs:79-158``) with the synthetic topologies;
``leo_b200_config_validate`` restates ``Config::validate``
(``crates/leo-core/src/config.rs:250-519``) plus the device limits;
``leo_b200_training_state_hash`` restates ``training_state_hash``
(``crates/leo-cli/src/main.rs:1151-1202``).  All three must agree with the
oracle byte for byte.
"""

from dataclasses import replace

import numpy as np
import pytest

from leo_b200.configs import BASELINE1, BASELINE2, PROBE, TEST
from leo_b200.ctypes_types import TOPOLOGY_REFERENCE, TOPOLOGY_UNIFORM, TOPOLOGY_ZIPF


@pytest.mark.parametrize("cfg_name,cfg,topology", [
    ("test-reference", TEST, TOPOLOGY_REFERENCE),
    ("test-uniform", TEST, TOPOLOGY_UNIFORM),
    ("test-zipf", TEST, TOPOLOGY_ZIPF),
    ("probe-reference", PROBE, TOPOLOGY_REFERENCE),
    ("baseline1-uniform", BASELINE1, TOPOLOGY_UNIFORM),
    ("baseline2-uniform", BASELINE2, TOPOLOGY_UNIFORM),
])
def test_initialize_matches_oracle(native_lib, oracle_lib, cfg_name, cfg, topology):
    from leo_b200.model import HostModel

    product = HostModel.initialize(cfg, topology)
    oracle = oracle_lib.OracleModel.initialize(cfg, topology)
    ref = oracle.arrays()
    for name, arr in product.arrays.items():
        assert arr.dtype == ref[name].dtype, name
        assert np.array_equal(arr.view(np.uint8), ref[name].view(np.uint8)), f"{cfg_name}: {name} differs"
    product.validate()
    oracle.validate()
    assert product.training_state_hash() == oracle.training_state_hash()


def test_initialize_is_seed_dependent(native_lib):
    from leo_b200.model import HostModel

    a = HostModel.initialize(TEST, TOPOLOGY_UNIFORM)
    b = HostModel.initialize(replace(TEST, seed=TEST.seed + 1), TOPOLOGY_UNIFORM)
    assert a.training_state_hash() != b.training_state_hash()
    assert not np.array_equal(a.arrays["recurrent_target"], b.arrays["recurrent_target"])


def test_weight_sign_rules(native_lib):
    """model.rs:362-379: excitatory sources never carry negative weights off
    the inhibitory branch; inhibitory sources only drive branch 1 with w <= 0."""
    from leo_b200.model import HostModel

    m = HostModel.initialize(BASELINE1, TOPOLOGY_UNIFORM)
    a = m.arrays
    S = BASELINE1.synapses_per_neuron
    src_type = np.repeat(a["neuron_type"], S)
    w, br = a["recurrent_weight"], a["recurrent_branch"]
    assert np.all(np.abs(w) <= 1.0)
    assert np.all(w[(src_type == 0)] >= 0.0)
    assert np.all(w[(src_type == 1)] <= 0.0)
    assert np.all(br[(src_type == 1)] == 1)
    assert set(np.unique(a["recurrent_delay"])) <= {1, 2, 4, 8}


INVALID = {
    "neuron_count_mismatch": dict(neuron_count=4095),
    "zero_blocks": dict(block_count=0),
    "keep_zero": dict(max_active_per_block=0),
    "decay_above_one": dict(membrane_decay=1.5),
    "negative_rate": dict(output_learning_rate=-0.1),
    "weight_bounds": dict(weight_min=1.0, weight_max=-1.0),
    "target_activity_above_cap": dict(target_activity=0.5),
    "context_order_zero": dict(context_max_order=0),
    "replay_fraction": dict(replay_fraction=1.5),
    "dropout_rate": dict(context_dropout_rate=1.5),
}


@pytest.mark.parametrize("name", sorted(INVALID))
def test_invalid_configs_rejected_by_both(native_lib, oracle_lib, name):
    import ctypes as C

    cfg = replace(PROBE, **INVALID[name])
    cc = cfg.to_c()
    assert native_lib.leo_b200_config_validate(C.byref(cc)) != 0
    assert oracle_lib.lib().leo_oracle_config_validate(C.byref(cc)) != 0
    assert native_lib.leo_b200_last_error()


@pytest.mark.parametrize("cfg", [TEST, PROBE, BASELINE1, BASELINE2], ids=["test", "probe", "baseline1", "baseline2"])
def test_valid_configs_accepted_by_both(native_lib, oracle_lib, cfg):
    import ctypes as C

    cc = cfg.to_c()
    assert native_lib.leo_b200_config_validate(C.byref(cc)) == 0
    assert oracle_lib.lib().leo_oracle_config_validate(C.byref(cc)) == 0


def test_device_limits_are_enforced(native_lib, oracle_lib):
    """Selection limits of the device path (the reference GPU's are at
    cuda.rs:9389-9437): block_count * keep <= 2048 block winners and at most
    1024 actives per tick.  The oracle has no such limits."""
    import ctypes as C

    ok = replace(PROBE, neuron_count=16384, block_count=256, neurons_per_block=64, max_active_per_block=8,
                 max_active_global=1024)
    for cfg, accepted in [(ok, True),
                          (replace(ok, max_active_per_block=9), False),
                          (replace(ok, neuron_count=65536, neurons_per_block=256, max_active_global=1025), False)]:
        cc = cfg.to_c()
        assert (native_lib.leo_b200_config_validate(C.byref(cc)) == 0) == accepted
        assert oracle_lib.lib().leo_oracle_config_validate(C.byref(cc)) == 0


def test_model_validate_catches_corruption(native_lib, oracle_lib):
    from leo_b200.model import HostModel

    m = HostModel.initialize(TEST, TOPOLOGY_REFERENCE)
    bad = m.copy()
    bad.arrays["recurrent_delay"][0] = 3
    from leo_b200.native import LeoError

    with pytest.raises(LeoError):
        bad.validate()
    with pytest.raises(RuntimeError):
        oracle_lib.OracleModel.from_arrays(TEST, bad.arrays).validate()
    bad = m.copy()
    bad.arrays["recurrent_target"][0] = TEST.neuron_count
    with pytest.raises(LeoError):
        bad.validate()
