"""Package shim mirroring the reference's ``cascade`` package
(cascade/__init__.py:1-16) on top of the B200 ``cascade_cpp``."""
from cascade_cpp import (CascadeConfig, CascadeStore, DistributedConfig, DistributedStore,
                         compute_block_id, compute_block_ids)

__all__ = ["CascadeStore", "CascadeConfig", "DistributedStore", "DistributedConfig",
           "compute_block_id", "compute_block_ids", "create_login_node_store",
           "compute_block_id_from_bytes"]


def create_login_node_store():
    """Small store (reference cascade/__init__.py:3-10). The reference's is
    CPU-only; here the 1 GiB DRAM-tier arena is filled by GPU copy kernels."""
    cfg = CascadeConfig()
    cfg.use_gpu = False
    cfg.shm_capacity_bytes = 1 * 1024 * 1024 * 1024
    cfg.shm_path = "/dev/shm/cascade_login"
    cfg.lustre_path = ""
    return CascadeStore(cfg)


def compute_block_id_from_bytes(data):
    """compute_block_id of a bytes object (reference cascade/__init__.py:12-16)."""
    import numpy as np
    return compute_block_id(np.frombuffer(data, dtype=np.uint8))
