"""Expert-parallel Kimi-Linear MoE decode layer (one process per GPU, NCCL).

The 256 routed experts are sharded evenly over the G ranks of a process group:
expert e lives on rank e // (E / G).  The router weights and the shared expert
are replicated.  Per layer every rank:

  1. routes its own tokens (``moe_router``: sigmoid, biased top-k, renormalised
     and scaled weights -- engine/klinear/router.py:47-85, the same kernel as
     the single-GPU layer);
  2. packs every (token, route) pair's hidden row for the rank that owns the
     route's expert (``ep_dispatch``): fixed-capacity slots per destination
     (tokens * top_k each, so nothing can overflow), the owner-local expert id
     carried in the row's tail, unused slots marked -1;
  3. exchanges the payloads with one equal-split ``all_to_all_single``;
  4. runs gate/up + SwiGLU and the down projection for the rows it received
     with its local expert bank (the grouped kernels read each local expert's
     weights once for all rows that use it and skip the empty slots);
  5. returns the outputs with a second equal-split ``all_to_all_single``;
  6. computes the shared expert on its own tokens and combines
     bf16(sum_r y_r * w_r, fp32 in route order) + y_shared
     (engine/klinear/moe.py:317-334, moe_combine.py:209-261) with
     ``ep_combine``, reading each route's output at the slot it was sent from.

No step reads a count on the host, so a step made of these layers can be
captured in one CUDA graph.  Every rank must run the layer on the same number
of tokens (the capacity of the exchange buffers depends on it).  The result
equals the single-GPU layer's (``moe.moe_forward``) up to the fp32 rounding of
the combine.  The arithmetic is delegated to a backend object (``CudaExperts``
by default: this library's kernels), so the dispatch and combine logic can also
run over ``gloo`` ranks on the CPU with a test backend.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops
from .moe import SHARED_TC_TOKENS, MoELayerWeights


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

    def dispatch(self, hidden: torch.Tensor, routed: torch.Tensor, per_rank: int, world: int,
                 capacity: int):
        """(payload bf16 [world*capacity + T, H+8], slots int32 [T*k]); the last
        T rows are the rank's own rows with the shared expert's local id."""
        return ops.ep_dispatch(hidden, routed, per_rank, world, capacity, shared_id=per_rank)

    def experts(self, payload: torch.Tensor, bank: LocalExpertBank) -> torch.Tensor:
        """Down(SwiGLU(gate/up)) of each payload row with its local expert, bf16 [n, H];
        rows of empty slots (id -1) are skipped and left undefined."""
        width = payload.shape[1] - 8
        rows = payload[:, :width]
        idx = ops.payload_ids(payload).contiguous()
        tc = self.use_tc(payload.shape[0], bank)
        swiglu = ops.w4a16_swiglu_tc if tc else ops.w4a16_swiglu
        grouped = ops.w4a16_grouped_tc if tc else ops.w4a16_grouped
        act = swiglu(rows, idx, bank.w1_packed, bank.w1_scales, bank.w3_packed, bank.w3_scales)
        return grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]

    @staticmethod
    def use_tc(slots: int, bank: LocalExpertBank) -> bool:
        """Tensor-core path for the received rows when the exchange buffer holds
        several rows per local expert on average (upper bound of the real load:
        the buffer includes empty slots): its units share each activation chunk
        across 256 weight rows, the engine restages it per 16."""
        if slots < 4 * bank.per_rank:
            return False
        h = bank.w1_packed.shape[2] * 2
        inter = bank.w1_packed.shape[1]
        return (ops.tc_supported(slots, inter, h, h // bank.w1_scales.shape[2])
                and ops.tc_supported(slots, h, inter, inter // bank.w2_scales.shape[2]))

    def shared(self, hidden: torch.Tensor, bank: LocalExpertBank) -> torch.Tensor:
        """The shared expert (local bank slot per_rank) on this rank's tokens, bf16 [T, H]."""
        t = hidden.shape[0]
        idx = torch.full((t, 1), bank.per_rank, dtype=torch.long, device=hidden.device)
        big = t >= SHARED_TC_TOKENS
        swiglu = ops.w4a16_swiglu_tc if big else ops.w4a16_swiglu
        grouped = ops.w4a16_grouped_tc if big else ops.w4a16_grouped
        act = swiglu(hidden, idx, bank.w1_packed, bank.w1_scales, bank.w3_packed,
                     bank.w3_scales)
        return grouped(act[:, 0], idx, bank.w2_packed, bank.w2_scales)[:, 0]

    def combine(self, y: torch.Tensor, slots: torch.Tensor, weights: torch.Tensor,
                shared: torch.Tensor) -> torch.Tensor:
        return ops.ep_combine(y, slots, weights, shared)


class ExpertParallelMoE:
    """One MoE layer with its experts sharded over ``group`` (the default
    process group when None).  ``forward`` takes this rank's tokens; every
    rank passes the same number of tokens."""

    def __init__(self, layer: MoELayerWeights, group=None, backend=None):
        self.group = group
        # Without a process group the layer runs on one GPU: the same data
        # plane with the exchanges reduced to identities and the bank used in
        # place.
        self.single = group is None and not (dist.is_available() and dist.is_initialized())
        self.rank = 0 if self.single else dist.get_rank(group)
        self.world = 1 if self.single else dist.get_world_size(group)
        self.layer = layer
        if self.world == 1:
            self.bank = LocalExpertBank(0, layer.num_experts, layer.w1_packed, layer.w1_scales,
                                        layer.w3_packed, layer.w3_scales, layer.w2_packed,
                                        layer.w2_scales)
        else:
            self.bank = shard_bank(layer, self.rank, self.world)
        self.backend = backend if backend is not None else CudaExperts()
        self.last_payload: torch.Tensor | None = None
        self.last_received: torch.Tensor | None = None

    def _exchange(self, tensor: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return tensor
        out = torch.empty_like(tensor)
        dist.all_to_all_single(out, tensor.contiguous(), group=self.group)
        return out

    def touched_local_experts(self) -> int:
        """Distinct local experts the last forward's received rows used (host read)."""
        if self.last_received is None:
            return 0
        ids = ops.payload_ids(self.last_received)[:, 0]
        routed = ids[(ids >= 0) & (ids < self.bank.per_rank)]
        return int(torch.unique(routed).numel())

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        """hidden bf16 [T, H] (this rank's tokens) -> bf16 [T, H]."""
        layer, bank, be = self.layer, self.bank, self.backend
        tokens, width = hidden.shape
        k = layer.top_k
        stable, weights = be.route(hidden, layer)
        routed = stable[:, :k]   # row-strided view; the dispatch kernel takes the stride
        capacity = max(1, tokens * k)
        n = self.world * capacity
        payload, slots = be.dispatch(hidden, routed, bank.per_rank, self.world, capacity)
        # The received rows, then this rank's own rows for the shared expert
        # (local bank slot per_rank): one gate/up and one down launch serve
        # both, so the shared expert's few row tiles do not run as launches of
        # their own on a fraction of the GPU.
        # A dispatch that already wrote the shared rows (after the slots)
        # returns n + tokens rows; otherwise they are appended here.
        own = payload.shape[0] >= n + tokens
        if self.world == 1:
            received = payload if own else torch.cat(
                (payload[:n], payload.new_empty((tokens, payload.shape[1]))))
        else:
            received = payload.new_empty((n + tokens, payload.shape[1]))
            dist.all_to_all_single(received[:n], payload[:n].contiguous(), group=self.group)
            if own:
                received[n:].copy_(payload[n:])
        if not own:
            received[n:, :width].copy_(hidden)
            ops.payload_ids(received[n:]).fill_(bank.per_rank)
        self.last_payload, self.last_received = payload[:n], received
        y_all = be.experts(received, bank)
        y_back = self._exchange(y_all[:n])
        return be.combine(y_back, slots, weights, y_all[n:])
