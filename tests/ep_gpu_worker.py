"""Run under torch.distributed.run, one rank per GPU (test_ep_gpu.py starts it): an expert-parallel decode block
(strata_mlx_b200/ep.py) against the single-device block on every rank's tokens, bit for bit. Exits non-zero on a
difference."""

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from strata_mlx_b200 import blocks as B  # noqa: E402
from strata_mlx_b200 import ep as EP  # noqa: E402
from strata_mlx_b200 import fused as F  # noqa: E402
from strata_mlx_b200.synthetic import layer_numpy  # noqa: E402

H, I, E, K, S = 2048, 512, 32, 10, 512


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    bad = 0
    chain_one, chain_par = [], []
    # more wrappers of the same layers (each with a workspace of its own): a chain of distinct layer objects whose
    # calls reuse each half of the exchange buffer within one step
    extra = []
    for kinds in (("IQ3_S", "IQ3_S", "Q2_0"), ("Q2_0", "Q2_0", "IQ3_XXS")):
        L = layer_numpy(np.random.default_rng(5), H, I, E, kinds, shared_inter=S)
        cu = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in L.items()
              if isinstance(v, np.ndarray) and v.dtype.kind in "fiu"}
        full = {k: B.BlockSwitchLinear(cu[k], kind, shp) for k, kind, shp in (
            ("gate", kinds[0], (E, I, H)), ("up", kinds[1], (E, I, H)), ("down", kinds[2], (E, H, I)))}
        shared = tuple(B.BlockSwitchLinear(cu[k], kind, shp) for k, kind, shp in (
            ("sgate", kinds[0], (1, S, H)), ("sup", kinds[1], (1, S, H)), ("sdown", kinds[2], (1, H, S))))
        e0, e1 = EP.expert_range(rank, world, E)
        mine = {k: B.BlockSwitchLinear(EP.local_experts(cu[k], E, rank, world), lin.kind,
                                       (e1 - e0, lin.output_dims, lin.input_dims))
                for k, lin in full.items()}
        one = F.MoEDecodeLayer(cu["router"], full["gate"], full["up"], full["down"], K, shared=shared,
                               shared_gate=cu["shared_gate"])
        par = EP.EPMoEDecodeLayer(cu["router"], mine["gate"], mine["up"], mine["down"], K, E, shared=shared,
                                  shared_gate=cu["shared_gate"])
        chain_one.append(one)
        chain_par.append(par)
        extra.append([EP.EPMoEDecodeLayer(cu["router"], mine["gate"], mine["up"], mine["down"], K, E, shared=shared,
                                          shared_gate=cu["shared_gate"]) for _ in range(2)])
        for t in (1, 2):
            x = torch.randn((t, H), generator=torch.Generator(device=dev).manual_seed(10 * rank + t), device=dev)
            x = x.to(torch.bfloat16)
            got = par(x)
            want = torch.cat([one(x[i : i + 1]) for i in range(t)])
            torch.cuda.synchronize()
            if not torch.equal(got, want):
                bad += 1
                diff = (got.float() - want.float()).abs().max().item()
                print(f"rank {rank} {kinds} t={t}: differs from the single-device block (max {diff})", flush=True)
    # the two layers as a chain with the exchange in the kernels (peer memory): three steps, so that the counts are
    # reset and reused across steps
    for t in (1, 2):
        chain = EP.EPDecodeChain(chain_par, t, dev)
        for step in range(3):
            x = torch.randn((t, H), generator=torch.Generator(device=dev).manual_seed(100 * step + 10 * rank + t),
                            device=dev).to(torch.bfloat16)
            got = chain(x).clone()
            want = x
            for one in chain_one:
                want = torch.cat([one(want[i : i + 1]) for i in range(t)])
            torch.cuda.synchronize()
            chain.check_errors()
            if not torch.equal(got, want):
                bad += 1
                diff = (got.float() - want.float()).abs().max().item()
                print(f"rank {rank} peer chain t={t} step {step}: differs (max {diff})", flush=True)
        dist.barrier()
        chain.close()
    # four layers fed again after two (refeed 2): the result is the last two layers on x, not all four in a row
    for t in (1, 2):
        chain = EP.EPDecodeChain([chain_par[0], chain_par[1], chain_par[1], chain_par[0]], t, dev)
        for step in range(2):
            x = torch.randn((t, H), generator=torch.Generator(device=dev).manual_seed(1000 + 100 * step + 10 * rank + t),
                            device=dev).to(torch.bfloat16)
            got = chain(x, refeed=2).clone()
            want = x
            for one in (chain_one[1], chain_one[0]):
                want = torch.cat([one(want[i : i + 1]) for i in range(t)])
            torch.cuda.synchronize()
            chain.check_errors()
            if not torch.equal(got, want):
                bad += 1
                diff = (got.float() - want.float()).abs().max().item()
                print(f"rank {rank} refed chain t={t} step {step}: differs (max {diff})", flush=True)
        dist.barrier()
        chain.close()
    # six distinct layer objects fed again every two layers: window halves and pair-output halves are reused by
    # other layers in the same step (their tags must still be this call's), the result the last two layers on x
    for t in (1, 2):
        chain = EP.EPDecodeChain([chain_par[0], chain_par[1], extra[0][0], extra[1][0], extra[0][1], extra[1][1]], t,
                                 dev)
        for step in range(3):
            x = torch.randn((t, H), generator=torch.Generator(device=dev).manual_seed(2000 + 100 * step + 10 * rank + t),
                            device=dev).to(torch.bfloat16)
            got = chain(x, refeed=2).clone()
            want = x
            for one in chain_one:
                want = torch.cat([one(want[i : i + 1]) for i in range(t)])
            torch.cuda.synchronize()
            chain.check_errors()
            if not torch.equal(got, want):
                bad += 1
                diff = (got.float() - want.float()).abs().max().item()
                print(f"rank {rank} six-layer chain t={t} step {step}: differs (max {diff})", flush=True)
        dist.barrier()
        chain.close()
    flag = torch.tensor([bad], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("ep bits: " + ("same" if flag.item() == 0 else f"{flag.item()} cases differ"), flush=True)
    sys.exit(1 if flag.item() else 0)


if __name__ == "__main__":
    main()
