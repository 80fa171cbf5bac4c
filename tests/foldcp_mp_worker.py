"""One rank of the multi-GPU Fold-CP parity check (launched by test_gpu_foldcp_multiproc.py
under torch.distributed.run): every rank runs the 2-block stack on its tile with each
transport ("peer": NVLink peer windows, "nccl": point-to-point batches) and compares the
gathered result with the single-device stack computed on its own GPU."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from opendde_b200.distributed.foldcp import clear_mesh_cache  # noqa: E402
from opendde_b200.model import PairformerStack  # noqa: E402
from opendde_b200.utils import ragged_pair_mask, seeded_init_  # noqa: E402


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def main():
    local = int(os.environ["LOCAL_RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    n = int(os.environ.get("FOLDCP_TEST_N", "300"))
    stack = PairformerStack(n_blocks=2, n_heads=16, c_z=128, c_s=384)
    seeded_init_(stack, seed=0)
    stack = stack.to(dev)
    g = torch.Generator().manual_seed(1)
    z = torch.randn((n, n, 128), generator=g).to(dev, torch.bfloat16)
    s = torch.randn((n, 384), generator=g).to(dev, torch.bfloat16)
    mask = ragged_pair_mask(n, seed=3, drop=0.2, full_rows=[5]).to(dev)
    os.environ["OPENDDE_FOLDCP_MODE"] = "single"
    with torch.no_grad():
        s1, z1 = stack(s, z, mask)
    os.environ.update({"OPENDDE_FOLDCP_MODE": "distributed", "OPENDDE_FOLDCP_SIZE_CP": str(world),
                       "OPENDDE_FOLDCP_SIZE_DP": "1"})
    worst = 0.0
    for transport in ("peer", "nccl"):
        os.environ["OPENDDE_B200_FOLDCP_TRANSPORT"] = transport
        with torch.no_grad():
            s2, z2 = stack(s, z, mask)
        torch.cuda.synchronize()
        ez, es = rel_l2(z2, z1), rel_l2(s2, s1)
        worst = max(worst, ez, es)
        print(f"rank {dist.get_rank()} {transport}: rel-L2 z {ez:.2e} s {es:.2e}", flush=True)
    t = torch.tensor([worst], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    clear_mesh_cache()
    dist.destroy_process_group()
    if t.item() > 5e-3:
        print(f"FAIL worst rel-L2 {t.item():.3e}", flush=True)
        sys.exit(1)
    print("OK", flush=True)


if __name__ == "__main__":
    main()
