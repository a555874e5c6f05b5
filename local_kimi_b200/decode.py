"""Kimi-Linear-48B-A3B W4A16 decode step on the B200 kernels (the hot path).

One decode step runs, for each of the 27 layers, every INT4 projection of the
layer, the KDA recurrent-state step of the KDA layers, and the MoE block
(router top-8 with the shared route appended, gate/up + SwiGLU over the
touched experts, down projection + routing-weighted combine), then the INT4
lm_head.  Shapes follow engine/klinear/config.py:38-80 (hidden 2304, 27 layers
with MLA at layers 4, 8, ..., 24, 27 one-based and KDA elsewhere, KDA 32 heads
x 128, MLA 32 heads with q 32 x 192 and kv_b 512 -> 32 x 256, 256 experts +
1 shared, intermediate 1024, layer 0 a dense 9216-wide MLP, vocab 163840) and
the INT4 classes of engine/quant/klinear_plan.py:320-419 (attention
projections, experts, shared expert, layer-0 MLP; plus the INT4 lm_head of
KLinearModel.quantize_lm_head, engine/klinear/model.py:134-160).

The parts of a layer that are not on this path -- RMS norms, the short
convolutions and gates that prepare the KDA inputs, MLA softmax attention, the
BF16-retained projections -- are not computed.  Their outputs enter as fixed
synthetic tensors: the KDA step reads fixed normalised q/k, v, decay and beta;
the MLA kv_b and o_proj projections read a fixed latent and attention output.
The data dependencies kept are the ones along the path: the KDA step output
(bf16) feeds o_proj, o_proj feeds the MoE block, the MoE output feeds the next
layer's projections, the last layer's output feeds the lm_head.

Weights are random-init (N(0, 0.02) bf16, quantised on the device by the
codec kernel), generated from seeded CUDA generators.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import ops
from .moe import MoELayerWeights, moe_forward
from .step import StepProgram


@dataclass(frozen=True)
class KimiLinearShape:
    vocab_size: int = 163_840
    hidden: int = 2_304
    layers: int = 27
    kda_heads: int = 32
    kda_head_dim: int = 128
    mla_heads: int = 32
    mla_q_head_dim: int = 192      # qk_nope 128 + qk_rope 64
    kv_lora_rank: int = 512
    mla_kv_head_dim: int = 256     # qk_nope 128 + v 128
    mla_v_head_dim: int = 128
    experts: int = 256
    top_k: int = 8
    moe_intermediate: int = 1_024
    dense_intermediate: int = 9_216
    routed_scaling_factor: float = 2.446
    first_k_dense: int = 1
    # one-based full-attention (MLA) layers, engine/klinear/config.py:10
    mla_layers: tuple[int, ...] = field(default_factory=lambda: (4, 8, 12, 16, 20, 24, 27))

    def is_mla(self, layer: int) -> bool:
        return (layer + 1) in self.mla_layers


@dataclass
class LayerWeights:
    kind: str                       # "kda" or "mla"
    qkv: list[tuple[torch.Tensor, torch.Tensor]] | None = None   # KDA q, k, v (views)
    # The three KDA projections stored as one [3 * C, K/2] matrix (q rows, then
    # k, then v); ``qkv`` holds row views of it.  Many-token steps project all
    # three in one tensor-core launch.
    qkv_fused: tuple[torch.Tensor, torch.Tensor] | None = None
    q_proj: tuple[torch.Tensor, torch.Tensor] | None = None      # MLA
    kv_b: tuple[torch.Tensor, torch.Tensor] | None = None        # MLA
    o_proj: tuple[torch.Tensor, torch.Tensor] | None = None
    kda_state: torch.Tensor | None = None                        # fp32 [B, H, 128, 128]
    moe: MoELayerWeights | None = None
    # KDA decode preparation: short-convolution weights and states of q, k, v
    # (bf16 [C, 4] and [B, C, 4]), dt_bias fp32 [C], A_log fp32 [H]
    conv_w: list[torch.Tensor] | None = None
    conv_state: list[torch.Tensor] | None = None
    dt_bias: torch.Tensor | None = None
    a_log: torch.Tensor | None = None
    dense_mlp: tuple | None = None  # (w1p, w1s, w3p, w3s) banks [1, I, H/2], (w2p, w2s)


def _bytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


class HotPathDecoder:
    """Synthetic-weight Kimi-Linear-48B-A3B decode hot path for a batch of B tokens."""

    def __init__(self, batch: int, *, group: int = 128, device: str | torch.device = "cuda",
                 shape: KimiLinearShape | None = None, seed: int = 0,
                 layers: int | None = None, kda_prepare: bool = True) -> None:
        # With kda_prepare the KDA inputs come from the layer's q/k/v
        # projections through the short convolutions and gates
        # (kb_kda_prepare); without it they are fixed synthetic tensors (the
        # decode-step executor's programs use those).
        self.kda_prepare = kda_prepare
        self.shape = shape or KimiLinearShape()
        self.batch = batch
        self.group = group
        self.device = torch.device(device)
        self.nlayers = self.shape.layers if layers is None else layers
        self._gen = torch.Generator(device=self.device)
        self._gen.manual_seed(seed)
        s = self.shape
        self.layers: list[LayerWeights] = []
        for layer in range(self.nlayers):
            self.layers.append(self._make_layer(layer))
        self.lm_head = self._quant(s.vocab_size, s.hidden)
        self._make_inputs(seed + 1)


    # -- weights ---------------------------------------------------------------
    def _randn(self, shape) -> torch.Tensor:
        return (torch.randn(shape, generator=self._gen, device=self.device) * 0.02).to(
            torch.bfloat16)

    def _quant(self, n: int, k: int) -> tuple[torch.Tensor, torch.Tensor]:
        return ops.quantise(self._randn((n, k)), self.group)

    def _bank(self, experts: int, n: int, k: int) -> tuple[torch.Tensor, torch.Tensor]:
        packed = torch.empty((experts, n, k // 2), dtype=torch.uint8, device=self.device)
        scales = torch.empty((experts, n, k // self.group), dtype=torch.bfloat16,
                             device=self.device)
        chunk = 64
        for e0 in range(0, experts, chunk):
            e1 = min(experts, e0 + chunk)
            p, sc = ops.quantise(self._randn(((e1 - e0) * n, k)), self.group)
            packed[e0:e1] = p.view(e1 - e0, n, k // 2)
            scales[e0:e1] = sc.view(e1 - e0, n, k // self.group)
        return packed, scales

    def _make_layer(self, layer: int) -> LayerWeights:
        s = self.shape
        B = self.batch
        if s.is_mla(layer):
            lw = LayerWeights(
                kind="mla",
                q_proj=self._quant(s.mla_heads * s.mla_q_head_dim, s.hidden),
                kv_b=self._quant(s.mla_heads * s.mla_kv_head_dim, s.kv_lora_rank),
                o_proj=self._quant(s.hidden, s.mla_heads * s.mla_v_head_dim),
            )
        else:
            proj = s.kda_heads * s.kda_head_dim
            parts = [self._quant(proj, s.hidden) for _ in range(3)]
            fused = (torch.cat([pk for pk, _ in parts]), torch.cat([sc for _, sc in parts]))
            del parts
            lw = LayerWeights(
                kind="kda",
                qkv=[(fused[0][i * proj:(i + 1) * proj], fused[1][i * proj:(i + 1) * proj])
                     for i in range(3)],
                qkv_fused=fused,
                o_proj=self._quant(s.hidden, proj),
                kda_state=0.05 * torch.randn((B, s.kda_heads, s.kda_head_dim, s.kda_head_dim),
                                             generator=self._gen, device=self.device),
                conv_w=[(0.3 * torch.randn((proj, 4), generator=self._gen,
                                           device=self.device)).to(torch.bfloat16)
                        for _ in range(3)],
                dt_bias=torch.randn(proj, generator=self._gen, device=self.device),
                a_log=torch.log(1.0 + 15.0 * torch.rand(s.kda_heads, generator=self._gen,
                                                        device=self.device)),
            )
            lw.conv_state = self._conv_states(B, self._gen)
        if layer < s.first_k_dense:
            w1 = self._bank(1, s.dense_intermediate, s.hidden)
            w3 = self._bank(1, s.dense_intermediate, s.hidden)
            w2 = self._quant(s.hidden, s.dense_intermediate)
            lw.dense_mlp = (w1, w3, w2)
        else:
            router = self._randn((s.experts, s.hidden))
            w1 = self._bank(s.experts + 1, s.moe_intermediate, s.hidden)
            w2 = self._bank(s.experts + 1, s.hidden, s.moe_intermediate)
            w3 = self._bank(s.experts + 1, s.moe_intermediate, s.hidden)
            lw.moe = MoELayerWeights(router, torch.zeros(s.experts, device=self.device), *w1,
                                     *w2, *w3, top_k=s.top_k, scaling=s.routed_scaling_factor)
        return lw

    def _conv_states(self, batch: int, gen: torch.Generator) -> list[torch.Tensor]:
        proj = self.shape.kda_heads * self.shape.kda_head_dim
        return [torch.randn((batch, proj, 4), generator=gen, device=self.device).to(
            torch.bfloat16) for _ in range(3)]

    def _make_inputs(self, seed: int) -> None:
        s = self.shape
        B = self.batch
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        self.x0 = torch.randn((B, s.hidden), generator=g, device=self.device).to(torch.bfloat16)
        H, D = s.kda_heads, s.kda_head_dim
        self.kda_q = F.normalize(torch.randn((B, H, D), generator=g, device=self.device), dim=-1)
        self.kda_k = F.normalize(torch.randn((B, H, D), generator=g, device=self.device), dim=-1)
        self.kda_v = 0.2 * torch.randn((B, H, D), generator=g, device=self.device)
        self.kda_decay = -(0.005 + 0.075 * torch.rand((B, H, D), generator=g,
                                                      device=self.device))
        self.kda_beta = torch.sigmoid(torch.randn((B, H), generator=g, device=self.device))
        self.kda_out = torch.empty((B, H * D), dtype=torch.bfloat16, device=self.device)
        # outputs of the BF16 gate projections (f_a/f_b and b_proj, not on the
        # INT4 path), fixed
        self.raw_decay = torch.randn((B, H * D), generator=g, device=self.device).to(
            torch.bfloat16)
        self.raw_beta = torch.randn((B, H), generator=g, device=self.device).to(torch.bfloat16)
        self.mla_latent = torch.randn((B, s.kv_lora_rank), generator=g,
                                      device=self.device).to(torch.bfloat16)
        self.mla_attn = torch.randn((B, s.mla_heads * s.mla_v_head_dim), generator=g,
                                    device=self.device).to(torch.bfloat16)
        self.dense_idx = torch.zeros((B, 1), dtype=torch.long, device=self.device)

    # -- batch views and expert parallelism -------------------------------------------
    def with_batch(self, batch: int, seed: int | None = None) -> "HotPathDecoder":
        """A decoder for ``batch`` tokens sharing this one's weights (no copy):
        new KDA states and synthetic inputs, the same quantised matrices."""
        import copy

        other = copy.copy(self)
        other.batch = batch
        g = torch.Generator(device=self.device)
        g.manual_seed(1000 + batch if seed is None else seed)
        s = self.shape
        other.layers = []
        for lw in self.layers:
            nl = copy.copy(lw)
            if lw.kda_state is not None:
                nl.kda_state = 0.05 * torch.randn(
                    (batch, s.kda_heads, s.kda_head_dim, s.kda_head_dim), generator=g,
                    device=self.device)
                nl.conv_state = self._conv_states(batch, g)
            other.layers.append(nl)
        other.ep_layers = None
        other._make_inputs((seed if seed is not None else 1) + 1)
        return other

    def enable_expert_parallel(self, group=None) -> None:
        """Run every MoE layer through ExpertParallelMoE over ``group`` (one
        process per GPU; without an initialised process group, one GPU).  The
        routed experts of a layer are sharded over the ranks; a rank keeps only
        its shard of each bank."""
        from .ep import ExpertParallelMoE

        self.ep_layers = {}
        for li, lw in enumerate(self.layers):
            if lw.moe is None:
                continue
            ep = ExpertParallelMoE(lw.moe, group=group)
            self.ep_layers[li] = ep
            if ep.world > 1:
                m = lw.moe
                # The full bank is no longer needed on this rank.
                lw.moe = MoELayerWeights(m.router_weight, m.router_bias, m.w1_packed[:0],
                                         m.w1_scales[:0], m.w2_packed[:0], m.w2_scales[:0],
                                         m.w3_packed[:0], m.w3_scales[:0], top_k=m.top_k,
                                         scaling=m.scaling)
                ep.layer = lw.moe
        torch.cuda.empty_cache()

    # -- one step --------------------------------------------------------------------
    def step(self, x: torch.Tensor, routes: list | None = None) -> torch.Tensor:
        """x bf16 [B, hidden] -> logits bf16 [B, vocab].  With ``routes`` (a
        list) the routed expert ids of every single-GPU MoE layer are appended."""
        s = self.shape
        eps = getattr(self, "ep_layers", None)
        for li, lw in enumerate(self.layers):
            if lw.kind == "kda":
                probs = [(x, *lw.qkv[0]), (x, *lw.qkv[1]), (x, *lw.qkv[2])]
                if lw.qkv_fused is not None and ops.multi_prefers_tc(probs):
                    # One launch over the three stacked matrices: enough row
                    # tiles to fill the GPU, then column views (one row stride).
                    n = lw.qkv[0][0].shape[0]
                    y = ops.w4a16_dense_tc(x, *lw.qkv_fused)
                    q_in, k_in, v_in = y[:, :n], y[:, n:2 * n], y[:, 2 * n:]
                else:
                    q_in, k_in, v_in = ops.w4a16_dense_multi(probs)
                fused = self.kda_prepare and ops.kda_prepare_step_supported(
                    lw.kda_state, s.kda_head_dim)
                if fused:
                    # Preparation and state step in one launch.
                    ops.kda_prepare_step(lw.kda_state, q_in, k_in, v_in, *lw.conv_state,
                                         *lw.conv_w, self.raw_decay, lw.dt_bias, lw.a_log,
                                         self.raw_beta, num_heads=s.kda_heads,
                                         head_dim=s.kda_head_dim,
                                         scale=s.kda_head_dim ** -0.5, out_bf16=self.kda_out)
                else:
                    if self.kda_prepare:
                        kin = ops.kda_prepare(q_in, k_in, v_in, *lw.conv_state, *lw.conv_w,
                                              self.raw_decay, lw.dt_bias, lw.a_log,
                                              self.raw_beta, num_heads=s.kda_heads,
                                              head_dim=s.kda_head_dim)
                    else:
                        kin = (self.kda_q, self.kda_k, self.kda_v, self.kda_decay,
                               self.kda_beta)
                    ops.kda_decode_step(lw.kda_state, *kin, scale=s.kda_head_dim ** -0.5,
                                        out_bf16=self.kda_out)
                h = ops.w4a16_dense(self.kda_out, *lw.o_proj)
            else:
                # q_proj and kv_b feed the attention, whose output feeds o_proj.
                ops.w4a16_dense_multi([(x, *lw.q_proj), (self.mla_latent, *lw.kv_b)])
                h = ops.w4a16_dense(self.mla_attn, *lw.o_proj)
            if lw.dense_mlp is not None:
                (w1p, w1s), (w3p, w3s), (w2p, w2s) = lw.dense_mlp
                tokens, hid = h.shape
                tc = ops.prefer_tc(tokens, w1p.shape[1], hid, hid // w1s.shape[2])
                swiglu = ops.w4a16_swiglu_tc if tc else ops.w4a16_swiglu
                act = swiglu(h, self.dense_idx, w1p, w1s, w3p, w3s)
                x = ops.w4a16_dense(act.view(h.shape[0], -1), w2p, w2s)
            elif eps is not None:
                x = eps[li].forward(h)
            else:
                x, idx, _ = moe_forward(h, lw.moe)
                if routes is not None:
                    routes.append(idx)
        return ops.w4a16_dense(x, *self.lm_head)

    @property
    def launches_per_step(self) -> int:
        return self._count_launches()

    def _count_launches(self) -> int:
        n = 1  # lm_head
        for lw in self.layers:
            n += 3 if lw.kind == "kda" else 2   # q/k/v, (preparation +) KDA step, o_proj
            n += 2 if lw.dense_mlp is not None else 3
        return n

    # -- the same step as one executor program ------------------------------------------
    def build_program(self, x: torch.Tensor) -> tuple[StepProgram, dict[str, object]]:
        """The step of ``step(x)`` as a decode-step executor program.

        Returns the finalized program and its buffers: ``logits`` (the
        output), ``idx``/``weights`` (routing of every MoE layer) and the
        intermediates.  Operations depend on the operations that produce their
        inputs as in the model (the KDA step on the q/k/v projections, MLA's
        o_proj on q_proj/kv_b, each layer on the previous layer's output).
        The program's KDA states are the layers' own states, as in ``step``.
        """
        s = self.shape
        B = self.batch
        dev = self.device
        bf = torch.bfloat16
        proj = s.kda_heads * s.kda_head_dim
        buf: dict[str, object] = {
            "x_in": x,
            "xa": torch.empty((B, s.hidden), dtype=bf, device=dev),
            "xb": torch.empty((B, s.hidden), dtype=bf, device=dev),
            "q": torch.empty((B, proj), dtype=bf, device=dev),
            "k": torch.empty((B, proj), dtype=bf, device=dev),
            "v": torch.empty((B, proj), dtype=bf, device=dev),
            "mla_q": torch.empty((B, s.mla_heads * s.mla_q_head_dim), dtype=bf, device=dev),
            "mla_kv": torch.empty((B, s.mla_heads * s.mla_kv_head_dim), dtype=bf, device=dev),
            "h": torch.empty((B, s.hidden), dtype=bf, device=dev),
            "act": torch.empty((B * (s.top_k + 1), s.moe_intermediate), dtype=bf, device=dev),
            "routed": torch.empty((B * (s.top_k + 1), s.hidden), dtype=bf, device=dev),
            "act0": torch.empty((B, s.dense_intermediate), dtype=bf, device=dev),
            "logits": torch.empty((B, s.vocab_size), dtype=bf, device=dev),
            "router_scratch": [], "idx": [], "weights": [],
        }
        prog = StepProgram(B)
        prev = None
        xin = x
        outs = [buf["xa"], buf["xb"]]
        for li, lw in enumerate(self.layers):
            xout = outs[li % 2]
            if lw.kind == "kda":
                qkv = prog.dense([(xin, *lw.qkv[0], buf["q"]), (xin, *lw.qkv[1], buf["k"]),
                                  (xin, *lw.qkv[2], buf["v"])], deps=[prev])
                kda = prog.kda(lw.kda_state, self.kda_q, self.kda_k, self.kda_v, self.kda_decay,
                               self.kda_beta, s.kda_head_dim ** -0.5, out_bf16=self.kda_out,
                               deps=[qkv])
                oproj = prog.dense([(self.kda_out, *lw.o_proj, buf["h"])], deps=[kda])
            else:
                qkvb = prog.dense([(xin, *lw.q_proj, buf["mla_q"]),
                                   (self.mla_latent, *lw.kv_b, buf["mla_kv"])], deps=[prev])
                oproj = prog.dense([(self.mla_attn, *lw.o_proj, buf["h"])], deps=[qkvb])
            if lw.dense_mlp is not None:
                (w1p, w1s), (w3p, w3s), (w2p, w2s) = lw.dense_mlp
                sw = prog.swiglu(buf["h"], (w1p[0], w1s[0]), (w3p[0], w3s[0]), buf["act0"],
                                 deps=[oproj])
                prev = prog.dense([(buf["act0"], w2p, w2s, xout)], deps=[sw])
            else:
                m = lw.moe
                lg = StepProgram.router_scratch(B, m.num_experts, dev)
                idx = torch.empty((B, m.top_k + 1), dtype=torch.long, device=dev)
                wts = torch.empty((B, m.top_k), dtype=torch.float32, device=dev)
                buf["router_scratch"].append(lg)
                buf["idx"].append(idx)
                buf["weights"].append(wts)
                r = prog.router(buf["h"], m.router_weight, m.router_bias, m.top_k, m.scaling, lg,
                                idx, wts, deps=[oproj])
                prev = prog.moe(r, buf["h"], m, buf["act"], buf["routed"], xout, deps=[oproj])
            xin = xout
        prog.dense([(xin, *self.lm_head, buf["logits"])], deps=[prev])
        return prog.finalize(), buf

    # -- byte accounting ----------------------------------------------------------------
    def weight_bytes(self) -> int:
        """Resident bytes of every quantised weight and bf16 router of the model."""
        total = _bytes(self.lm_head[0]) + _bytes(self.lm_head[1])
        for lw in self.layers:
            for pair in (lw.qkv or []) + [m for m in (lw.q_proj, lw.kv_b, lw.o_proj) if m]:
                total += _bytes(pair[0]) + _bytes(pair[1])
            if lw.dense_mlp is not None:
                total += sum(_bytes(t) for pair in lw.dense_mlp for t in pair)
            if lw.moe is not None:
                m = lw.moe
                total += sum(_bytes(t) for t in (m.router_weight, m.w1_packed, m.w1_scales,
                                                 m.w2_packed, m.w2_scales, m.w3_packed,
                                                 m.w3_scales))
        return total

    def step_bytes(self, expert_counts: list[int] | None = None) -> dict[str, int]:
        """Algorithmic bytes of one step by component.

        expert_counts[l]: distinct experts (routed + shared) touched in MoE
        layer l; defaults to top_k + 1 per token capped at E + 1 (batch 1).
        """
        s = self.shape
        B = self.batch
        out = {"dense_proj": 0, "experts": 0, "router": 0, "kda_state": 0, "lm_head": 0,
               "activations": 0}
        moe_i = 0
        for lw in self.layers:
            mats = (lw.qkv or []) + [m for m in (lw.q_proj, lw.kv_b, lw.o_proj) if m is not None]
            for p, sc in mats:
                out["dense_proj"] += _bytes(p) + _bytes(sc)
            if lw.kda_state is not None:
                out["kda_state"] += 2 * _bytes(lw.kda_state)
                if self.kda_prepare:
                    # conv states read and written, q/k/v in, five fp32 outputs
                    out["kda_state"] += sum(2 * _bytes(c) for c in lw.conv_state)
            if lw.dense_mlp is not None:
                (w1p, w1s), (w3p, w3s), (w2p, w2s) = lw.dense_mlp
                out["dense_proj"] += sum(_bytes(t) for t in (w1p, w1s, w3p, w3s, w2p, w2s))
            if lw.moe is not None:
                m = lw.moe
                per_expert = (sum(_bytes(t[0]) for t in (m.w1_packed, m.w1_scales, m.w2_packed,
                                                         m.w2_scales, m.w3_packed, m.w3_scales))
                              if m.w1_packed.shape[0] else 0)  # bank sharded away
                touched = (expert_counts[moe_i] if expert_counts is not None
                           else min(s.experts + 1, B * s.top_k + 1))
                out["experts"] += per_expert * touched
                out["router"] += _bytes(m.router_weight)
                moe_i += 1
        out["lm_head"] = _bytes(self.lm_head[0]) + _bytes(self.lm_head[1])
        out["activations"] = B * s.hidden * 2 * (2 * self.nlayers) + B * s.vocab_size * 2
        out["total"] = sum(out.values())
        return out

    def touched_experts(self, x: torch.Tensor) -> list[int]:
        """Distinct experts (routed + shared) per MoE layer for input x: one
        step run eagerly with every recurrent state put back afterwards."""
        saved = [(lw.kda_state.clone(), [c.clone() for c in lw.conv_state])
                 for lw in self.layers if lw.kda_state is not None]
        routes: list[torch.Tensor] = []
        self.step(x, routes=routes)
        for lw, (st, conv) in zip([lw for lw in self.layers if lw.kda_state is not None], saved):
            lw.kda_state.copy_(st)
            for c, c0 in zip(lw.conv_state, conv):
                c.copy_(c0)
        return [int(torch.unique(idx).numel()) + 1 for idx in routes]
