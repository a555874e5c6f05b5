"""Expert-parallel Kimi-Linear MoE decode layer (one process per GPU, NCCL).

The 256 routed experts are sharded evenly over the G ranks of a process group:
expert e lives on rank e // (E / G).  The router weights and the shared expert
are replicated.  Per layer every rank:

  1. routes its own tokens (``moe_router``: sigmoid, biased top-k, renormalised
     and scaled weights -- engine/klinear/router.py:47-85, the same kernel as
     the single-GPU layer);
  2. sends each (token, route) pair's hidden row to the rank that owns the
     route's expert, ordered by destination (stable, so token-major then route
     order inside each destination): first the per-destination counts
     (``all_to_all_single`` of int64 [G]), then the rows and the owner-local
     expert ids with exact split sizes (no capacity padding; the counts are
     read on the host once per layer);
  3. runs gate/up + SwiGLU and the down projection for the rows it received
     with its local expert bank (the grouped kernels, which read each local
     expert's weights once for all rows that use it);
  4. returns the per-route outputs to their source ranks with the reverse
     ``all_to_all_single``;
  5. computes the shared expert on its own tokens and combines
     bf16(sum_r y_r * w_r, fp32 in route order) + y_shared
     (engine/klinear/moe.py:317-334, moe_combine.py:209-261) with
     ``moe_combine_routes``.

The result equals the single-GPU layer's (``moe.moe_forward``) up to the fp32
rounding of the combine.  The arithmetic is delegated to a backend object
(``CudaExperts`` by default: this library's kernels), so the dispatch and
combine logic can also run over ``gloo`` ranks on the CPU with a test backend.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops
from .moe import MoELayerWeights


@dataclass
class LocalExpertBank:
    """This rank's experts: local slot j < per_rank is global expert first + j,
    slot per_rank is the shared expert (global bank slot E)."""

    first: int
    per_rank: int
    w1_packed: torch.Tensor
    w1_scales: torch.Tensor
    w3_packed: torch.Tensor
    w3_scales: torch.Tensor
    w2_packed: torch.Tensor
    w2_scales: torch.Tensor


def shard_bank(layer: MoELayerWeights, rank: int, world: int) -> LocalExpertBank:
    """Slices rank ``rank``'s experts (and the shared expert) out of a full bank."""
    experts = layer.num_experts
    if experts % world:
        raise ValueError(f"{experts} experts do not divide evenly over {world} ranks")
    per = experts // world
    first = rank * per
    sel = torch.cat((torch.arange(first, first + per), torch.tensor([experts]))).to(
        layer.w1_packed.device
    )

    def take(t: torch.Tensor) -> torch.Tensor:
        return t.index_select(0, sel).contiguous()

    return LocalExpertBank(first, per, take(layer.w1_packed), take(layer.w1_scales),
                           take(layer.w3_packed), take(layer.w3_scales),
                           take(layer.w2_packed), take(layer.w2_scales))


class CudaExperts:
    """The arithmetic of the expert-parallel layer on this library's kernels."""

    def route(self, hidden: torch.Tensor, layer: MoELayerWeights):
        """(indices int64 [T, k+1] with the shared expert id E last, weights fp32 [T, k])."""
        return ops.moe_router(hidden, layer.router_weight, layer.router_bias, layer.top_k,
                              routed_scaling_factor=layer.scaling,
                              append_expert=layer.num_experts)

    def experts(self, rows: torch.Tensor, local_ids: torch.Tensor,
                bank: LocalExpertBank) -> torch.Tensor:
        """Down(SwiGLU(gate/up)) of each row with its local expert, bf16 [n, H]."""
        idx = local_ids.view(-1, 1)
        act = ops.w4a16_swiglu(rows, idx, bank.w1_packed, bank.w1_scales, bank.w3_packed,
                               bank.w3_scales)
        return ops.w4a16_grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]

    def combine(self, routes: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        return ops.moe_combine_routes(routes, weights)


class ExpertParallelMoE:
    """One MoE layer with its experts sharded over ``group`` (the default
    process group when None).  ``forward`` takes this rank's tokens."""

    def __init__(self, layer: MoELayerWeights, group=None, backend=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.layer = layer
        self.bank = shard_bank(layer, self.rank, self.world)
        self.backend = backend if backend is not None else CudaExperts()
        self.last_counts: tuple[list[int], list[int]] | None = None

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, out_split: list[int],
                  in_split: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_split, in_split, group=self.group)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        """hidden bf16 [T, H] (this rank's tokens) -> bf16 [T, H]."""
        layer, bank, be = self.layer, self.bank, self.backend
        tokens, width = hidden.shape
        k = layer.top_k
        stable, weights = be.route(hidden, layer)
        routed = stable[:, :k].reshape(-1)
        dest = torch.div(routed, bank.per_rank, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=self.world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_split = send_counts.tolist()
        recv_split = recv_counts.tolist()
        self.last_counts = (send_split, recv_split)
        send_rows = hidden.index_select(0, torch.div(order, k, rounding_mode="floor"))
        send_ids = routed[order] - dest[order] * bank.per_rank
        recv_rows = hidden.new_empty((sum(recv_split), width))
        recv_ids = send_ids.new_empty((sum(recv_split),))
        self._exchange(recv_rows, send_rows, recv_split, send_split)
        self._exchange(recv_ids, send_ids, recv_split, send_split)
        y_recv = be.experts(recv_rows, recv_ids, bank)
        y_send = hidden.new_empty((tokens * k, width))
        self._exchange(y_send, y_recv.contiguous(), send_split, recv_split)
        y_routed = hidden.new_empty((tokens * k, width))
        y_routed[order] = y_send
        shared_ids = torch.full((tokens,), bank.per_rank, dtype=torch.int64,
                                device=hidden.device)
        y_shared = be.experts(hidden, shared_ids, bank)
        routes = torch.cat((y_routed.view(tokens, k, width), y_shared.view(tokens, 1, width)),
                           dim=1)
        return be.combine(routes, weights)
