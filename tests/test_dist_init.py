"""init_expert_parallel: the NCCL settings are in the environment before the process
group exists, explicit user settings win, and the group has the launcher's rank and size
(gloo ranks on CPU)."""
import os
import sys
from pathlib import Path

import numpy as np
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _worker(rank, ws, rdzv, out_dir):
    sys.path.insert(0, str(ROOT))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(ws), LOCAL_RANK=str(rank), NCCL_BUFFSIZE="123")
    for k in ("NCCL_P2P_LEVEL", "NCCL_NVLS_ENABLE"):
        os.environ.pop(k, None)
    import torch.distributed as dist
    import swiftmoe_b200 as S
    seen = {}
    real = dist.init_process_group

    def spy(*a, **kw):          # what the environment holds when the group is created
        seen.update(p2p=os.environ.get("NCCL_P2P_LEVEL"), nvls=os.environ.get("NCCL_NVLS_ENABLE"),
                    buf=os.environ.get("NCCL_BUFFSIZE"))
        return real(*a, **kw)

    dist.init_process_group = spy
    r, n, local = S.init_expert_parallel("gloo", nvls=False, init_method=f"file://{rdzv}", timeout_s=30)
    again = S.init_expert_parallel("gloo")             # a second call changes nothing
    ok = (r == rank and n == ws and local == rank and again == (r, n, local) and seen["p2p"] == "NVL"
          and seen["nvls"] == "0" and seen["buf"] == "123")
    np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array([float(ok)]))
    dist.barrier()
    dist.destroy_process_group()


def test_init_expert_parallel_applies_settings_before_the_group(tmp_path):
    mp.spawn(_worker, args=(2, str(tmp_path / "rdzv"), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert float(np.load(tmp_path / f"ok{r}.npy")[0]) == 1.0
