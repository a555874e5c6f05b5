"""CPU restatements of the hot-path operators (test oracle, not product code).

Each function cites the reference it restates.  Decoded weights are
bf16(code * scale) (engine/kernels/w4a16_gemv.py:146-158,
engine/quant/triton_w4a16.py:105-113); products and sums run in fp32 on the
CPU; every projection output is rounded to bf16 (w4a16_gemv.py:533-539).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .codec import decode_bf16


def dense(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """x[M,K] . dequant(W[N,K])^T -> bf16 [M,N]  (registry op w4a16_dense,
    engine/kernels/__init__.py:92-125; the same test oracle as
    tests/test_w4a16_dense_gemv.py:7-22 with bf16-rounded decode)."""
    w = decode_bf16(packed, scales)
    return F.linear(x.float(), w).to(torch.bfloat16)


def grouped(
    x: torch.Tensor, idx: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor
) -> torch.Tensor:
    """y[t,r] = x[t] . dequant(W[idx[t,r]])^T -> bf16 [T,R,N]
    (engine/kernels/w4a16_grouped.py:121-194, w4a16_gemv.py:610-635)."""
    t, r = idx.shape
    n = packed.shape[1]
    out = torch.empty((t, r, n), dtype=torch.bfloat16)
    xf = x.float()
    for e in torch.unique(idx).tolist():
        tok, route = torch.where(idx == e)
        w = decode_bf16(packed[e], scales[e])
        out[tok, route] = F.linear(xf[tok], w).to(torch.bfloat16)
    return out


def swiglu(
    x: torch.Tensor,
    idx: torch.Tensor,
    w1p: torch.Tensor,
    w1s: torch.Tensor,
    w3p: torch.Tensor,
    w3s: torch.Tensor,
) -> torch.Tensor:
    """F.silu(grouped(w1)) * grouped(w3) in bf16 (engine/kernels/__init__.py:182-197)."""
    gate = grouped(x, idx, w1p, w1s)
    up = grouped(x, idx, w3p, w3s)
    return F.silu(gate) * up


def w2_combine(
    activated: torch.Tensor,
    idx: torch.Tensor,
    weights: torch.Tensor,
    w2p: torch.Tensor,
    w2s: torch.Tensor,
    *,
    return_parts: bool = False,
):
    """Down projection of every route + combine (engine/kernels/moe_combine.py:209-261).

    ``weights`` has R columns (last ignored) or R-1 columns (routed only).
    With ``return_parts`` also returns the bf16 routed sum and shared output
    whose bf16 sum is the result.
    """
    t, r, k = activated.shape
    outputs = torch.empty((t, r, w2p.shape[1]), dtype=torch.bfloat16)
    for route in range(r):
        outputs[:, route] = grouped(activated[:, route], idx[:, route : route + 1], w2p, w2s)[:, 0]
    routed = (
        outputs[:, : r - 1].float().mul(weights[:, : r - 1].float().unsqueeze(-1)).sum(dim=1)
    ).to(torch.bfloat16)
    out = routed + outputs[:, r - 1]
    if return_parts:
        return out, combine_rounding_bound(outputs, weights, routed)
    return out


def bf16_spacing(values: torch.Tensor) -> torch.Tensor:
    """Distance between adjacent bf16 numbers at |values| (8 significant bits)."""
    m = values.float().abs().clamp_min(torch.finfo(torch.float32).tiny)
    return torch.exp2(torch.floor(torch.log2(m)) - 7)


def combine_rounding_bound(outputs: torch.Tensor, weights: torch.Tensor,
                           routed: torch.Tensor) -> torch.Tensor:
    """One bf16 spacing of every rounded term the combined output is built from.

    out = bf16(sum_r w_r y_r) + y_shared, each y_r a bf16-rounded dot product.
    An implementation whose fp32 sums differ from this oracle's only in order
    may land each rounded term on the neighbouring bf16 value; this bound is
    the sum of those spacings (weighted by |w_r| for the routed terms).  It
    matters only where routed and shared cancel.
    """
    r = outputs.shape[1]
    bound = bf16_spacing(routed) + bf16_spacing(outputs[:, r - 1])
    bound = bound + (weights[:, : r - 1].float().abs().unsqueeze(-1)
                     * bf16_spacing(outputs[:, : r - 1])).sum(dim=1)
    return bound


def fused_qkv(x, qp, qs, kp, ks, vp, vs):
    """Three dense projections (engine/kernels/w4a16_fused_qkv.py:257-271)."""
    return dense(x, qp, qs), dense(x, kp, ks), dense(x, vp, vs)


def router_logits(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp32 logits (engine/klinear/router.py:51)."""
    return F.linear(hidden.reshape(-1, hidden.shape[-1]).float(), weight.float())


def router_logits_lanes(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp32 logits (engine/klinear/router.py:51) summed in one fixed, stated order.

    The reference's F.linear leaves the order of the fp32 sum to the BLAS.
    This restatement fixes it to the order the B200 router kernels use, so
    that their logits -- and with them the top-k indices -- can be compared
    bit for bit:

    * the row of K bf16 values is cut into 16-byte words of 8 values; word w
      belongs to lane w mod 32 of a 32-lane group, and each lane visits its
      words in increasing order;
    * a lane keeps four partial sums, one per value pair j of a word; values
      2j and 2j+1 are added to partial j in that order (each bf16 x bf16
      product is exact in fp32, so a fused multiply-add is one rounded add);
    * the lane's total is (p0 + p1) + (p2 + p3);
    * the 32 lane totals are combined by a butterfly: lane l adds lane
      l xor 16, then l xor 8, 4, 2, 1; the result is lane 0's value.
    """
    h = hidden.reshape(-1, hidden.shape[-1]).float()
    w = weight.float()
    t, k = h.shape
    e = w.shape[0]
    words = k // 8
    per_lane = -(-words // 32)
    pad = per_lane * 32 * 8 - k
    if pad:
        h = F.pad(h, (0, pad))
        w = F.pad(w, (0, pad))
    # [T or E, per_lane, 32 lanes, 4 pairs, 2 values]
    hv = h.view(t, per_lane, 32, 4, 2)
    wv = w.view(e, per_lane, 32, 4, 2)
    out = torch.empty((t, e), dtype=torch.float32)
    for ti in range(t):
        prod = hv[ti].unsqueeze(0) * wv                       # exact in fp32
        acc = torch.zeros((e, 32, 4), dtype=torch.float32)
        for i in range(per_lane):
            acc = acc + prod[:, i, :, :, 0]
            acc = acc + prod[:, i, :, :, 1]
        lane = (acc[..., 0] + acc[..., 1]) + (acc[..., 2] + acc[..., 3])   # [E, 32]
        idx = torch.arange(32)
        for o in (16, 8, 4, 2, 1):
            lane = lane + lane[:, idx ^ o]
        out[ti] = lane[:, 0]
    return out


def router_topk(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    top_k: int,
    *,
    renormalize: bool = True,
    scaling: float = 1.0,
    logits: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sigmoid top-k with ties broken by the lower index (engine/klinear/router.py:47-85).

    The reference calls torch.topk(sorted=False), whose tie order is
    unspecified; this restatement orders by (choice desc, index asc) with a
    stable sort.  Returns (indices [T,k] in that order, weights [T,k] fp32,
    choice scores [T,E]).
    """
    lg = router_logits(hidden, weight) if logits is None else logits
    scores = lg.sigmoid()
    choice = scores + (bias.float().unsqueeze(0) if bias is not None else 0.0)
    order = torch.sort(choice, dim=-1, descending=True, stable=True).indices
    idx = order[:, :top_k]
    w = scores.gather(1, idx)
    if top_k > 1 and renormalize:
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
    return idx, w * scaling, choice


def shape_stable_indices(idx: torch.Tensor, shared_id: int) -> torch.Tensor:
    """Append the shared expert as the last route (engine/klinear/moe.py:23-36)."""
    shared = torch.full((idx.shape[0], 1), shared_id, dtype=idx.dtype)
    return torch.cat((idx, shared), dim=1)


def kda_step(
    state: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    decay: torch.Tensor,
    beta: torch.Tensor,
    *,
    scale: float,
) -> torch.Tensor:
    """KDA recurrence, mutating ``state`` (engine/kernels/kda_step.py:173-196)."""
    candidate = state * torch.exp(decay).unsqueeze(-1)
    prediction = (candidate * k.unsqueeze(-1)).sum(dim=-2)
    delta = v - prediction
    candidate = candidate + (beta.unsqueeze(-1).unsqueeze(-1) * k.unsqueeze(-1) * delta.unsqueeze(-2))
    output = (candidate * (q * scale).unsqueeze(-1)).sum(dim=-2)
    state.copy_(candidate)
    return output
