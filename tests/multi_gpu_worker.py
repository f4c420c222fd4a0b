"""One rank of the multi-GPU golden check (run by tests/test_multi_gpu.py under
torchrun): sharded story batches over NCCL must reproduce the single-GPU golden
training_state_hash on every rank."""

import datetime
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE / "golden"))


def main() -> int:
    import torch
    import torch.distributed as dist

    from make_golden import case_stories

    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel
    from leo_b200.parallel import TorchExchange, sharded_story_batch

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    host = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))
    ex = TorchExchange(None, host)
    golden = json.loads((HERE / "golden" / "story_batches.json").read_text())
    failures = []
    for name in sys.argv[1:]:
        case = {c["name"]: c for c in golden["cases"]}[name]
        w = WORKLOADS[case["workload"]]
        model = HostModel.initialize(w.config, w.topology)
        with GpuBackend(model, device=local, max_lanes=case["stories_per_batch"]) as gpu:
            for b, batch in enumerate(case_stories(case)):
                sharded_story_batch(gpu, ex, batch, TRAINING)
                if gpu.state_digest().hex() != case["batches"][b]["state_hash"]:
                    failures.append(f"{name} batch {b} rank {dist.get_rank()}")
    flag = torch.tensor([len(failures)], device=f"cuda:{local}")
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    for f in failures:
        print("MISMATCH", f, flush=True)
    return 1 if int(flag.item()) else 0


if __name__ == "__main__":
    raise SystemExit(main())
