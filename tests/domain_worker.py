"""Worker for ``test_domain_decomposition_equals_single_gpu`` (launched by torch.distributed.run)."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from ubio_molfm_b200.domain import domain_energy_forces  # noqa: E402
from ubio_molfm_b200.model import E2FormerPotential  # noqa: E402
from ubio_molfm_b200.synthetic import bio_box, seeded_params_  # noqa: E402


def main():
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl")
    dev = torch.device("cuda", local)
    cfg = dict(irreps_node_embedding="128x0e+128x1e+128x2e", num_layers=2, max_neighbors=24, max_radius=5.0,
               number_of_basis=32, num_attn_heads=16, attn_scalar_head=8, irreps_head="2x0e+2x1e+2x2e",
               norm_layer="rms_norm_sh", alpha_drop=0.0, avg_degree=23.0)
    m = E2FormerPotential(**cfg)
    seeded_params_(m, 5)
    m = m.to(dev).eval()
    pos, Z, cell = bio_box(1200, seed=4)
    pos = torch.tensor(pos, dtype=torch.float32, device=dev)
    Z = torch.tensor(Z, device=dev)
    cell = torch.tensor(cell, dtype=torch.float32)
    e_ref, f_ref = m(pos, Z, cell, (True, True, True))
    e, own, f = domain_energy_forces(m, pos, Z, cell)
    f_all = torch.zeros_like(f_ref)
    f_all[own] = f
    dist.all_reduce(f_all)
    de = abs(e.item() - e_ref.item()) / len(Z)
    df = (f_all - f_ref).abs().max().item()
    if rank == 0:
        print(f"energy {e.item():.6f} ref {e_ref.item():.6f} per-atom diff {de:.3e}; max force diff {df:.3e}")
        ok = de <= 1e-6 * abs(e_ref.item() / len(Z)) + 1e-7 and df <= 1e-4
        print("DOMAIN_OK" if ok else "DOMAIN_MISMATCH")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
