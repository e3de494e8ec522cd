"""One rank of the DHT failure-detection check (tests/test_gpu_dht.py, one
process per GPU, NCCL_NVLS_ENABLE=0). Both ranks put a batch; rank 1 then
leaves between steps (no kernel or collective in flight) and rank 0's next
collective get must end, within the short collective timeout, with
CB_ERR_TIMEOUT (or the NCCL error of the aborted peer), not hang."""
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cascade_cpp  # noqa: E402
from cascade_cpp import _lib as L  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    rank = dist.get_rank()
    cfg = cascade_cpp.DistributedConfig()
    cfg.gpu_capacity_per_device = 256 << 20
    cfg.dram_capacity = 0
    cfg.device = local
    cfg.collective_timeout_ms = 3000
    store = cascade_cpp.DistributedStore(cfg)
    rng = np.random.default_rng(rank)
    blocks = [torch.from_numpy(rng.integers(0, 256, 65536, dtype=np.uint8)).to(f"cuda:{local}") for _ in range(16)]
    ids = store.batch_put(blocks)
    store.barrier()
    torch.cuda.synchronize()
    if rank == 1:
        print("rank 1: leaving between steps", flush=True)
        os._exit(0)  # no destructor: the peer learns of it only through its next collective
    time.sleep(1.0)
    outs = [torch.empty(65536, dtype=torch.uint8, device=f"cuda:{local}") for _ in ids]
    t0 = time.perf_counter()
    try:
        store.batch_get(ids, outs)
    except cascade_cpp.CascadeError as e:
        dt = time.perf_counter() - t0
        assert e.code in (L.CB_ERR_TIMEOUT, L.CB_ERR_NCCL), e
        assert dt < 30.0, dt
        print(f"rank 0: collective failed after {dt:.1f} s with code {e.code}: {e}", flush=True)
        os._exit(0)
    print("rank 0: the get did not fail", flush=True)
    os._exit(1)


if __name__ == "__main__":
    main()
