"""Expert-parallel MoE layer (local_kimi_b200.ep).

CPU: two ``gloo`` ranks run the dispatch / expert / return / combine logic
with the oracle's arithmetic and must reproduce the single-process oracle
layer (oracle/moe.py) on the same tokens exactly.  GPU: the combine kernel
against the oracle combine, a one-rank NCCL layer against the single-GPU
layer, and (with two or more GPUs) two NCCL ranks against it.  Tolerance for
GPU results: 2e-2 relative or 1e-3 absolute per element (tests/conftest.py).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from local_kimi_b200.ep import ExpertParallelMoE, shard_bank
from local_kimi_b200.moe import MoELayerWeights
from oracle import codec
from oracle import moe as omoe
from oracle import ops as oref

E, H, I, TOP_K, GROUP = 8, 64, 32, 2, 32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bank(seed: int = 0):
    """A small seeded MoE bank (CPU), as MoELayerWeights and oracle MoEBanks."""
    g = torch.Generator().manual_seed(seed)

    def q(rows: int, cols: int):
        w = (0.02 * torch.randn((rows, cols), generator=g)).to(torch.bfloat16)
        p, s = codec.quantise(w, GROUP)
        return p, s

    def bank(n: int, k: int):
        ps = [q(n, k) for _ in range(E + 1)]
        return torch.stack([p for p, _ in ps]), torch.stack([s for _, s in ps])

    w1p, w1s = bank(I, H)
    w3p, w3s = bank(I, H)
    w2p, w2s = bank(H, I)
    router = (0.05 * torch.randn((E, H), generator=g)).to(torch.bfloat16)
    bias = 0.01 * torch.randn((E,), generator=g)
    layer = MoELayerWeights(router, bias, w1p, w1s, w2p, w2s, w3p, w3s, top_k=TOP_K,
                            scaling=2.446)
    banks = omoe.MoEBanks(router, bias, w1p, w1s, w2p, w2s, w3p, w3s, top_k=TOP_K,
                          scaling=2.446)
    return layer, banks


def _tokens(world: int, per_rank: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1)
    return torch.randn((world * per_rank, H), generator=g).to(torch.bfloat16)


class OracleExperts:
    """The layer's arithmetic restated by the oracle (test backend)."""

    def route(self, hidden, layer):
        idx, w, _ = oref.router_topk(hidden, layer.router_weight, layer.router_bias,
                                     layer.top_k, scaling=layer.scaling)
        return oref.shape_stable_indices(idx, layer.num_experts), w

    def experts(self, rows, local_ids, bank):
        idx = local_ids.view(-1, 1)
        act = oref.swiglu(rows, idx, bank.w1_packed, bank.w1_scales, bank.w3_packed,
                          bank.w3_scales)
        return oref.grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]

    def combine(self, routes, weights):
        r = routes.shape[1]
        routed = (routes[:, : r - 1].float() * weights[:, : r - 1].float().unsqueeze(-1)).sum(
            dim=1).to(torch.bfloat16)
        return routed + routes[:, r - 1]


def _cpu_rank(rank: int, world: int, port: int, per_rank: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer, banks = _bank()
        x = _tokens(world, per_rank)
        mine = x[rank * per_rank:(rank + 1) * per_rank]
        ep = ExpertParallelMoE(layer, backend=OracleExperts())
        out = ep.forward(mine)
        expected, idx, _ = omoe.moe_layer(x, banks)
        exp_mine = expected[rank * per_rank:(rank + 1) * per_rank]
        assert torch.equal(out, exp_mine), f"rank {rank}: EP output differs from the oracle"
        # every (token, route) pair went to the owner of its expert
        send, recv = ep.last_counts
        owners = torch.div(idx[rank * per_rank:(rank + 1) * per_rank], E // world,
                           rounding_mode="floor")
        assert send == torch.bincount(owners.reshape(-1), minlength=world).tolist()
        assert sum(recv) == int(
            (torch.div(idx, E // world, rounding_mode="floor") == rank).sum())
    finally:
        dist.destroy_process_group()


def test_shard_bank_slices_owned_experts_and_shared():
    layer, _ = _bank()
    b = shard_bank(layer, 1, 2)
    assert b.first == 4 and b.per_rank == 4
    assert torch.equal(b.w1_packed[:4], layer.w1_packed[4:8])
    assert torch.equal(b.w2_scales[4], layer.w2_scales[E])
    with pytest.raises(ValueError):
        shard_bank(layer, 0, 3)


@pytest.mark.timeout(300)
def test_expert_parallel_two_gloo_ranks_match_oracle():
    mp.spawn(_cpu_rank, args=(2, _free_port(), 6), nprocs=2, join=True)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------


def _gpu_layer(device: str):
    layer, banks = _bank()
    moved = MoELayerWeights(*(t.to(device) if t is not None else None for t in (
        layer.router_weight, layer.router_bias, layer.w1_packed, layer.w1_scales,
        layer.w2_packed, layer.w2_scales, layer.w3_packed, layer.w3_scales)),
        top_k=layer.top_k, scaling=layer.scaling)
    return moved, banks


def _gpu_rank(rank: int, world: int, port: int, per_rank: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device(dev))
    try:
        from local_kimi_b200.moe import moe_forward
        from tests.conftest import assert_close

        layer, _ = _gpu_layer(dev)
        x = _tokens(world, per_rank).to(dev)
        mine = x[rank * per_rank:(rank + 1) * per_rank].contiguous()
        ep = ExpertParallelMoE(layer)
        for _ in range(2):
            out = ep.forward(mine)
        torch.cuda.synchronize()
        single, _, _ = moe_forward(mine, layer)
        assert_close(out, single.cpu(), what=f"EP rank {rank} vs single GPU")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_combine_routes_matches_oracle(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    from tests.conftest import assert_close
    from local_kimi_b200 import ops

    routes = torch.randn((37, 9, 2304), generator=g, device=cuda).to(torch.bfloat16)
    w = torch.rand((37, 8), generator=g, device=cuda)
    out = ops.moe_combine_routes(routes, w)
    assert_close(out, OracleExperts().combine(routes.cpu(), w.cpu()), what="combine routes")
    assert torch.equal(out, ops.moe_combine_routes(routes, w)), "combine not deterministic"


@pytest.mark.gpu
@pytest.mark.timeout(300)
def test_expert_parallel_one_nccl_rank_matches_single_gpu(cuda):
    mp.spawn(_gpu_rank, args=(1, _free_port(), 5), nprocs=1, join=True)


@pytest.mark.gpu
@pytest.mark.timeout(300)
def test_expert_parallel_two_nccl_ranks_match_single_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_gpu_rank, args=(2, _free_port(), 5), nprocs=2, join=True)
