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

from local_kimi_b200 import ops
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
    """The layer's arithmetic and data plane restated on the CPU (test backend)."""

    def route(self, hidden, layer):
        idx, w, _ = oref.router_topk(hidden, layer.router_weight, layer.router_bias,
                                     layer.top_k, scaling=layer.scaling)
        return oref.shape_stable_indices(idx, layer.num_experts), w

    def dispatch(self, hidden, routed, per_rank, world, capacity):
        # Pairs in token-major order; each takes the next free slot of its
        # destination rank (the stable scan of kb_ep_dispatch).
        t, h = hidden.shape
        k = routed.shape[1]
        payload = torch.zeros((world * capacity, h + 8), dtype=torch.bfloat16)
        ids = ops.payload_ids(payload)
        ids.fill_(-1)
        fill = [0] * world
        slots = torch.empty((t * k,), dtype=torch.int32)
        for a in range(t * k):
            tok, r = divmod(a, k)
            e = int(routed[tok, r])
            d = e // per_rank
            slot = d * capacity + fill[d]
            fill[d] += 1
            payload[slot, :h] = hidden[tok]
            ids[slot, 0] = e - d * per_rank
            slots[a] = slot
        return payload, slots

    def experts(self, payload, bank):
        h = payload.shape[1] - 8
        ids = ops.payload_ids(payload)[:, 0]
        out = torch.zeros((payload.shape[0], h), dtype=torch.bfloat16)
        valid = (ids >= 0).nonzero()[:, 0]
        if valid.numel():
            idx = ids[valid].view(-1, 1)
            act = oref.swiglu(payload[valid, :h], idx, bank.w1_packed, bank.w1_scales,
                              bank.w3_packed, bank.w3_scales)
            out[valid] = oref.grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]
        return out

    def shared(self, hidden, bank):
        idx = torch.full((hidden.shape[0], 1), bank.per_rank, dtype=torch.long)
        act = oref.swiglu(hidden, idx, bank.w1_packed, bank.w1_scales, bank.w3_packed,
                          bank.w3_scales)
        return oref.grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]

    def combine(self, y, slots, weights, shared):
        t, k = weights.shape
        routes = y[slots.long()].view(t, k, -1)
        routed = (routes.float() * weights.float().unsqueeze(-1)).sum(dim=1).to(torch.bfloat16)
        return routed + shared


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
        # every (token, route) pair went to the owner of its expert: the
        # filled slots of each destination block match the pairs it owns
        capacity = per_rank * TOP_K
        ids = ops.payload_ids(ep.last_payload)[:, 0]
        owners = torch.div(idx[rank * per_rank:(rank + 1) * per_rank], E // world,
                           rounding_mode="floor")
        sent = [(ids[d * capacity:(d + 1) * capacity] >= 0).sum().item() for d in range(world)]
        assert sent == torch.bincount(owners.reshape(-1), minlength=world).tolist()
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
    rc, wc = routes.cpu(), w.cpu()
    routed = (rc[:, :8].float() * wc.unsqueeze(-1)).sum(dim=1).to(torch.bfloat16)
    assert_close(out, routed + rc[:, 8], what="combine routes")
    assert torch.equal(out, ops.moe_combine_routes(routes, w)), "combine not deterministic"


@pytest.mark.gpu
@pytest.mark.parametrize("world,tokens", [(1, 64), (4, 17), (8, 32)])
def test_dispatch_and_combine_kernels_match_cpu_restatement(cuda, world, tokens):
    # kb_ep_dispatch against the CPU restatement of the slot layout (rows,
    # ids, empty slots, pair slots), then kb_ep_combine on returned outputs.
    from tests.conftest import assert_close

    g = torch.Generator().manual_seed(world * 100 + tokens)
    experts, k, h = 256, 8, 2304
    per_rank = experts // world
    hidden = torch.randn((tokens, h), generator=g).to(torch.bfloat16)
    routed = torch.stack([torch.randperm(experts, generator=g)[:k] for _ in range(tokens)])
    cap = tokens * k
    payload, slots = ops.ep_dispatch(hidden.to(cuda), routed.to(cuda), per_rank, world, cap)
    ref_payload, ref_slots = OracleExperts().dispatch(hidden, routed, per_rank, world, cap)
    ids = ops.payload_ids(payload).cpu()
    assert torch.equal(ids, ops.payload_ids(ref_payload))
    assert torch.equal(slots.cpu(), ref_slots)
    used = (ids[:, 0] >= 0).nonzero()[:, 0]
    assert torch.equal(payload.cpu()[used, :h], ref_payload[used, :h])
    y = torch.randn((world * cap, h), generator=g).to(torch.bfloat16)
    w = torch.rand((tokens, k), generator=g)
    shared = torch.randn((tokens, h), generator=g).to(torch.bfloat16)
    out = ops.ep_combine(y.to(cuda), slots, w.to(cuda), shared.to(cuda))
    assert_close(out, OracleExperts().combine(y, ref_slots, w, shared), what="ep combine")
    # With a shared-expert id the same slots, then every token's row once more
    # with that id.
    p2, s2 = ops.ep_dispatch(hidden.to(cuda), routed.to(cuda), per_rank, world, cap,
                             shared_id=per_rank)
    assert p2.shape[0] == world * cap + tokens
    assert torch.equal(s2.cpu(), ref_slots)
    ids2 = ops.payload_ids(p2).cpu()
    assert torch.equal(ids2[:world * cap], ops.payload_ids(ref_payload))
    assert bool((ids2[world * cap:, 0] == per_rank).all())
    assert torch.equal(p2.cpu()[world * cap:, :h], hidden)
    assert torch.equal(p2.cpu()[used, :h], ref_payload[used, :h])


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", [64, 200])
def test_single_gpu_expert_parallel_layer_matches_oracle(cuda, tokens):
    # The layer without a process group (one GPU: the same data plane with the
    # exchanges as identities) at decode widths, where the received rows run
    # on the tensor-core path, against the oracle layer.
    from local_kimi_b200.ep import CudaExperts
    from local_kimi_b200.moe import MoELayerWeights as W
    from tests.conftest import assert_close
    from tests.gpu_util import cuda_gen, quant_bank, rand_act, rand_weight

    gen = cuda_gen(600 + tokens)
    experts, hid, inter = 16, 2304, 1024
    w1 = quant_bank(experts + 1, inter, hid, 128, gen)
    w2 = quant_bank(experts + 1, hid, inter, 128, gen)
    w3 = quant_bank(experts + 1, inter, hid, 128, gen)
    router = rand_weight((experts, hid), gen)
    bias = 0.01 * torch.randn(experts, generator=gen, device=cuda)
    layer = W(router, bias, *w1, *w2, *w3, top_k=4, scaling=2.446)
    ep = ExpertParallelMoE(layer)
    assert ep.world == 1 and CudaExperts.use_tc(tokens * 4, ep.bank)
    x = rand_act((tokens, hid), gen)
    out = ep.forward(x)
    banks = omoe.MoEBanks(router.cpu(), bias.cpu(), w1[0].cpu(), w1[1].cpu(), w2[0].cpu(),
                          w2[1].cpu(), w3[0].cpu(), w3[1].cpu(), top_k=4, scaling=2.446)
    ref, idx, _, bound = omoe.moe_layer(x.cpu(), banks, return_parts=True, lane_order=True)
    assert_close(out, ref, what=f"single-GPU EP layer T={tokens}", allowance=bound)


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
