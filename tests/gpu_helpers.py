"""Run this package's CUDA modules and the CPU oracle on the same seeded inputs."""
import torch

from oracle import pairformer_oracle as O
from opendde_b200.utils import seeded_init_


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def max_abs(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def cuda_module(mod, params, device):
    with torch.no_grad():
        for n, p in mod.named_parameters():
            p.copy_(params[n])
    return mod.to(device)


def oracle_op(kind, s, z, mask, params):
    with torch.no_grad():
        if kind == "trimul_out":
            return O.triangle_multiplication(z, mask, params, outgoing=True)
        if kind == "trimul_in":
            return O.triangle_multiplication(z, mask, params, outgoing=False)
        if kind == "triatt_start":
            return O.triangle_attention(z, mask, params, 4, starting=True)
        if kind == "triatt_end":
            return O.triangle_attention(z, mask, params, 4, starting=False)
        if kind == "transition":
            return O.transition(z, params)
        if kind == "apb":
            return O.attention_pair_bias(s, z, params, 16)
        raise ValueError(kind)


def cuda_op(kind, mod, s, z, mask, device, dtype):
    zz = z.to(device=device, dtype=dtype)
    mm = mask.to(device)
    with torch.no_grad():
        if kind.startswith("trimul"):
            return mod(zz, mask=mm).float().cpu()
        if kind.startswith("triatt"):
            return mod(zz, mask=mm).float().cpu()
        if kind == "transition":
            return mod(zz).float().cpu()
        if kind == "apb":
            return mod(a=s.to(device=device, dtype=dtype), s=None, z=zz).float().cpu()
    raise ValueError(kind)
