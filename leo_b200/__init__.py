"""leo_b200: B200-native per-byte training step over Leo's logical story workers.

The package holds the sm_100a CUDA kernels and C++ host runtime (``csrc/``,
built in-tree into ``libleo_b200.so`` by :mod:`leo_b200.build`), the generated
kernel ABI (:mod:`leo_b200.abi`), and a Python host mirroring the reference's
backend contract (:mod:`leo_b200.backend`), its multi-GPU story sharding
(:mod:`leo_b200.parallel`), the ``PSCLS100`` checkpoints of the synchronized
model (:mod:`leo_b200.checkpoint`) and the ``LEODATA1`` dataset feed
(:mod:`leo_b200.dataset`).
"""

from .configs import WORKLOADS, Config, Workload  # noqa: F401
from .ctypes_types import FROZEN, PROVISIONAL, TRAINING, VERIFIED  # noqa: F401
