#!/usr/bin/env python
"""Decode-throughput benchmark of the Kimi-Linear-48B-A3B W4A16 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--total-batch B] [--impl b200|reference]

The benchmark step (every N, one process per GPU under torchrun) is one decode
step of the hot path (local_kimi_b200.decode) for B = 256 concurrent sequences
in total, B/N per rank, with random-init weights of the real shapes (about
25 GB, resident in HBM): for all 27 layers the INT4 attention projections and
the KDA recurrent-state step on the rank's own sequences, every MoE layer
expert-parallel over the N ranks (local_kimi_b200.ep: 256/N routed experts per
rank, fixed-capacity dispatch, NCCL all-to-all over NVLink, shared expert and
combine on the owning rank), then the INT4 lm_head.  N = 1 runs the same step
with all experts local.  The step is captured as one CUDA graph (eager
launches where capture is unavailable).

Printed: one JSON line.  ``value`` = tokens/s over all ranks (B / step time,
device-timed, max over ranks; strong scaling: B is fixed as N grows);
``e2e`` = the same with a host->device copy of the step input and a
device->host copy of the logits inside the timed region; ``roofline`` =
algorithmic bytes of rank 0's step over its time against the measured HBM
copy bandwidth; ``cpu_baseline`` = the oracle on a bounded sample of the same
step (BatchCpuSample, median of 10 after 3 warm-ups).  At N = 1 the line also
carries ``bs1`` (the batch-1 step on the one-launch decode-step executor, with
the per-operation graph and their logits compared), ``bs32`` (batch 32,
per-operation graph) and ``dense_sweep`` (the C2 sweep at M 1/16/64).  Every
step reads GBs of weights and KDA state, far more than the 126 MB L2, so no L2
flush is needed between steps.

``--impl reference`` times the reference's CPU path restated in ``oracle/``
(the reference is pure Python/torch and does not exist on the GPU box) on all
host cores, on the same bounded per-step sample, and prints the same metric.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "decode tok/s Kimi-Linear-48B W4A16 (hot path step)"
HBM_FALLBACK_GBS = 6650.0


def _args() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1, help="token count of the single-case runs")
    ap.add_argument("--total-batch", type=int, default=256,
                    help="sequences of the benchmark step over all ranks")
    ap.add_argument("--no-sweep", action="store_true",
                    help="leave the dense-sweep sub-record out of the N=1 line")
    ap.add_argument("--headline-only", action="store_true",
                    help="only the benchmark step (no sub-records, no CPU baseline)")
    ap.add_argument("--profile-step", action="store_true",
                    help="after the timing, run one eager benchmark step between "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--group", type=int, default=128)
    ap.add_argument("--layers", type=int, default=None, help="fewer layers (testing only)")
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--path", choices=("executor", "per-op"), default="executor",
                    help="executor: the whole step in one persistent launch (batch <= 8); "
                         "per-op: the registry-level launches captured in a CUDA graph")
    ap.add_argument("--case",
                    choices=("step", "lm_head", "moe", "eager", "program", "dense_sweep",
                             "ep_moe", "moe_layers", "kda", "experts"),
                    default="step",
                    help="step = the benchmark; the others run one op family eagerly for "
                         "profiling (lm_head: the INT4 lm_head GEMV; moe: router + experts + "
                         "combine of one layer; eager: uncaptured decode steps); "
                         "dense_sweep: the W4A16 dense GEMV/GEMM sweep (M 1/4/16/64 over the "
                         "QKV, o_proj, shared gate|up and lm_head shapes), HBM GB/s vs peak; "
                         "ep_moe: one MoE layer with its experts sharded over the torchrun "
                         "ranks, --batch tokens in total split over them (NCCL all-to-all); "
                         "moe_layers: router + gate/up + down/combine of distinct MoE layers "
                         "back to back in one graph (--zipf S skews the expert popularity); "
                         "kda: the KDA state step of --batch sequences (32 heads of 128x128); "
                         "experts: the routed-expert gate/up+SwiGLU and down tensor-core "
                         "launches of one MoE layer for --batch tokens (top-8 of 256 experts, "
                         "uniform random routes, as the expert-parallel step at one GPU)")
    ap.add_argument("--wide-sweep", action="store_true",
                    help="dense_sweep: also the MLA and dense-MLP shapes, both paths at every M")
    ap.add_argument("--zipf", type=float, default=0.0,
                    help="moe_layers: router bias giving expert e of a seeded permutation "
                         "popularity ~ rank^-S (0: unskewed)")
    return ap.parse_args()


def _peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML while running."""

    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int, period: float = 0.02) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self.period = period
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._nvml = None

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = int(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = statistics.median(s[0] for s in self.samples)
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = [name for name, bit in self.REASONS.items() if seen & bit]
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def _dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# ---------------------------------------------------------------------------
# CPU baseline: the oracle on a bounded sample of the step
# ---------------------------------------------------------------------------


class CpuSample:
    """CPU tensors for one KDA+MoE layer, one MLA+MoE layer, the dense layer 0
    and 1/8 of the lm_head rows, from the GPU model or generated on the CPU."""

    LM_HEAD_FRACTION = 8

    def __init__(self, batch: int, group: int, model=None, seed: int = 0) -> None:
        from local_kimi_b200.decode import KimiLinearShape
        from oracle import codec, synth

        s = model.shape if model is not None else KimiLinearShape()
        self.shape, self.batch, self.group = s, batch, group
        B, H, D = batch, s.kda_heads, s.kda_head_dim
        proj = H * D
        if model is not None:
            self.x = model.x0.cpu()
            self.q, self.k, self.v = model.kda_q.cpu(), model.kda_k.cpu(), model.kda_v.cpu()
            self.decay, self.beta = model.kda_decay.cpu(), model.kda_beta.cpu()
            self.latent, self.attn = model.mla_latent.cpu(), model.mla_attn.cpu()
            kl = next(lw for lw in model.layers if lw.kind == "kda" and lw.moe is not None)
            ml = next(lw for lw in model.layers if lw.kind == "mla")
            self.qkv = [(p.cpu(), sc.cpu()) for p, sc in kl.qkv]
            self.kda_o = tuple(t.cpu() for t in kl.o_proj)
            self.state = kl.kda_state.cpu()
            self.mla_q = tuple(t.cpu() for t in ml.q_proj)
            self.kv_b = tuple(t.cpu() for t in ml.kv_b)
            self.mla_o = tuple(t.cpu() for t in ml.o_proj)
            self._moe_src = {"kda": kl.moe, "mla": ml.moe}
            l0 = model.layers[0].dense_mlp
            self.dense = [t.cpu() for pair in l0 for t in pair]
            rows = s.vocab_size // self.LM_HEAD_FRACTION
            self.lm_head = (model.lm_head[0][:rows].cpu(), model.lm_head[1][:rows].cpu())
            self.n_kda = sum(1 for lw in model.layers if lw.kind == "kda" and lw.moe is not None)
            self.n_mla = sum(1 for lw in model.layers if lw.kind == "mla")
        else:
            gen = synth.generator(seed)
            act = synth.generator(seed + 1)
            self.x = synth.activations((B, s.hidden), act)
            self.q = torch.nn.functional.normalize(torch.randn((B, H, D), generator=act), dim=-1)
            self.k = torch.nn.functional.normalize(torch.randn((B, H, D), generator=act), dim=-1)
            self.v = 0.2 * torch.randn((B, H, D), generator=act)
            self.decay = -(0.005 + 0.075 * torch.rand((B, H, D), generator=act))
            self.beta = torch.sigmoid(torch.randn((B, H), generator=act))
            self.latent = synth.activations((B, s.kv_lora_rank), act)
            self.attn = synth.activations((B, s.mla_heads * s.mla_v_head_dim), act)
            q = lambda n, k: synth.quantised(n, k, group, gen)  # noqa: E731
            self.qkv = [q(proj, s.hidden) for _ in range(3)]
            self.kda_o = q(s.hidden, proj)
            self.state = 0.05 * torch.randn((B, H, D, D), generator=gen)
            self.mla_q = q(s.mla_heads * s.mla_q_head_dim, s.hidden)
            self.kv_b = q(s.mla_heads * s.mla_kv_head_dim, s.kv_lora_rank)
            self.mla_o = q(s.hidden, s.mla_heads * s.mla_v_head_dim)
            self._moe_src = {"kda": None, "mla": None}
            self._gen = gen
            w1, w3 = q(s.dense_intermediate, s.hidden), q(s.dense_intermediate, s.hidden)
            w2 = q(s.hidden, s.dense_intermediate)
            self.dense = [w1[0][None], w1[1][None], w3[0][None], w3[1][None], w2[0], w2[1]]
            self.lm_head = q(s.vocab_size // self.LM_HEAD_FRACTION, s.hidden)
            self.n_kda = sum(1 for i in range(s.layers) if not s.is_mla(i)) - s.first_k_dense
            self.n_mla = sum(1 for i in range(s.layers) if s.is_mla(i))
        self.codec = codec

    def moe_banks(self, kind: str, hidden: torch.Tensor):
        """Oracle banks holding exactly the experts this hidden state routes to."""
        from oracle import moe as omoe
        from oracle import ops as oref
        from oracle import synth

        s = self.shape
        m = self._moe_src[kind]
        if m is not None:
            router, bias = m.router_weight.cpu(), m.router_bias.cpu()
        else:
            router, bias = synth.weight((s.experts, s.hidden), self._gen), torch.zeros(s.experts)
        idx, _, _ = oref.router_topk(hidden, router, bias, s.top_k,
                                     scaling=s.routed_scaling_factor)
        used = torch.unique(torch.cat((idx.flatten(), torch.tensor([s.experts]))))
        dims = {0: (s.moe_intermediate, s.hidden), 1: (s.hidden, s.moe_intermediate),
                2: (s.moe_intermediate, s.hidden)}
        banks = []
        for j in range(3):
            n, k = dims[j]
            p = torch.zeros((s.experts + 1, n, k // 2), dtype=torch.uint8)
            sc = torch.zeros((s.experts + 1, n, k // self.group), dtype=torch.bfloat16)
            if m is not None:
                srcp = (m.w1_packed, m.w2_packed, m.w3_packed)[j]
                srcs = (m.w1_scales, m.w2_scales, m.w3_scales)[j]
                p[used] = srcp[used.to(srcp.device)].cpu()
                sc[used] = srcs[used.to(srcs.device)].cpu()
            else:
                for e in used.tolist():
                    p[e], sc[e] = synth.quantised(n, k, self.group, self._gen)
            banks += [p, sc]
        return omoe.MoEBanks(router, bias, *banks, s.top_k, s.routed_scaling_factor)

    def seconds_per_step(self) -> tuple[float, str, int]:
        from oracle import moe as omoe
        from oracle import ops as oref

        torch.set_num_threads(os.cpu_count() or 1)
        s, B = self.shape, self.batch
        scale = s.kda_head_dim ** -0.5
        # Routing inputs of the sampled layers (computed before timing).
        st = self.state.clone()
        o = oref.kda_step(st, self.q, self.k, self.v, self.decay, self.beta, scale=scale)
        h_kda = oref.dense(o.reshape(B, -1).to(torch.bfloat16), *self.kda_o)
        banks_kda = self.moe_banks("kda", h_kda)
        h_mla = oref.dense(self.attn, *self.mla_o)
        banks_mla = self.moe_banks("mla", h_mla)

        t0 = time.perf_counter()
        oref.fused_qkv(self.x, *self.qkv[0], *self.qkv[1], *self.qkv[2])
        st = self.state.clone()
        o = oref.kda_step(st, self.q, self.k, self.v, self.decay, self.beta, scale=scale)
        h = oref.dense(o.reshape(B, -1).to(torch.bfloat16), *self.kda_o)
        omoe.moe_layer(h, banks_kda)
        t_kda = time.perf_counter() - t0

        t0 = time.perf_counter()
        oref.dense(self.x, *self.mla_q)
        oref.dense(self.latent, *self.kv_b)
        h = oref.dense(self.attn, *self.mla_o)
        omoe.moe_layer(h, banks_mla)
        t_mla = time.perf_counter() - t0

        t0 = time.perf_counter()
        d = self.dense
        a = oref.swiglu(self.x, torch.zeros((B, 1), dtype=torch.long), d[0], d[1], d[2], d[3])
        oref.dense(a.view(B, -1), d[4], d[5])
        t_dense = time.perf_counter() - t0

        t0 = time.perf_counter()
        oref.dense(self.x, *self.lm_head)
        t_head = (time.perf_counter() - t0) * self.LM_HEAD_FRACTION

        total = t_kda * self.n_kda + t_mla * self.n_mla + t_dense + t_head
        sample = (f"oracle (torch CPU, {torch.get_num_threads()} threads) on 1 KDA+MoE layer, "
                  f"1 MLA+MoE layer, the dense layer 0 and 1/{self.LM_HEAD_FRACTION} of the "
                  f"lm_head rows at batch {B}; per-step time extrapolated to {self.n_kda} "
                  f"KDA+MoE + {self.n_mla} MLA+MoE layers + layer 0 + the full lm_head")
        return total, sample, torch.get_num_threads()


class BatchCpuSample:
    """The oracle (torch CPU, all cores) on a bounded sample of the batch decode
    step: one KDA attention block, one MLA attention block, one MoE layer, the
    dense MLP of layer 0 and 1/8 of the lm_head rows, at ``batch`` tokens.

    The MoE layer routes all tokens but computes the routed experts for only
    ``expert_sample`` of the experts it touches (each with its own tokens),
    scaled by the number touched; the shared expert runs on every token.  The
    KDA state step runs at ``kda_batch`` sequences and is scaled by
    batch / kda_batch (its cost is linear in the batch).  Weights are seeded
    synthetic values with the real shapes (the timing does not depend on the
    values); the per-step time is extrapolated to the 27-layer step.
    """

    LM_HEAD_FRACTION = 8

    def __init__(self, batch: int, group: int, seed: int = 0, expert_sample: int = 8,
                 kda_batch: int = 32) -> None:
        from local_kimi_b200.decode import KimiLinearShape
        from oracle import synth

        s = KimiLinearShape()
        self.shape, self.batch, self.group = s, batch, group
        self.expert_sample = expert_sample
        self.kda_batch = min(kda_batch, batch)
        gen = synth.generator(seed)
        act = synth.generator(seed + 1)
        H, D = s.kda_heads, s.kda_head_dim
        proj = H * D
        q = lambda n, k: synth.quantised(n, k, group, gen)  # noqa: E731
        self.x = synth.activations((batch, s.hidden), act)
        self.attn = synth.activations((batch, s.mla_heads * s.mla_v_head_dim), act)
        self.latent = synth.activations((batch, s.kv_lora_rank), act)
        self.kda_in = synth.activations((batch, proj), act)
        kb = self.kda_batch
        self.q = torch.nn.functional.normalize(torch.randn((kb, H, D), generator=act), dim=-1)
        self.k = torch.nn.functional.normalize(torch.randn((kb, H, D), generator=act), dim=-1)
        self.v = 0.2 * torch.randn((kb, H, D), generator=act)
        self.decay = -(0.005 + 0.075 * torch.rand((kb, H, D), generator=act))
        self.beta = torch.sigmoid(torch.randn((kb, H), generator=act))
        self.state = 0.05 * torch.randn((kb, H, D, D), generator=gen)
        self.conv_w = [synth.activations((proj, 4), gen) for _ in range(3)]
        self.conv_state = [synth.activations((batch, proj, 4), act) for _ in range(3)]
        self.raw_decay = synth.activations((batch, proj), act)
        self.raw_beta = synth.activations((batch, H), act)
        self.dt_bias = torch.randn(proj, generator=gen)
        self.a_log = torch.log(1.0 + 15.0 * torch.rand(H, generator=gen))
        self.qkv = [q(proj, s.hidden) for _ in range(3)]
        self.kda_o = q(s.hidden, proj)
        self.mla_q = q(s.mla_heads * s.mla_q_head_dim, s.hidden)
        self.kv_b = q(s.mla_heads * s.mla_kv_head_dim, s.kv_lora_rank)
        self.mla_o = q(s.hidden, s.mla_heads * s.mla_v_head_dim)
        self.router = synth.weight((s.experts, s.hidden), gen)
        self.experts = [(q(s.moe_intermediate, s.hidden), q(s.moe_intermediate, s.hidden),
                         q(s.hidden, s.moe_intermediate)) for _ in range(expert_sample + 1)]
        w1, w3 = q(s.dense_intermediate, s.hidden), q(s.dense_intermediate, s.hidden)
        w2 = q(s.hidden, s.dense_intermediate)
        self.dense = (w1, w3, w2)
        self.lm_head = q(s.vocab_size // self.LM_HEAD_FRACTION, s.hidden)
        self.n_kda = sum(1 for i in range(s.layers) if not s.is_mla(i))
        self.n_mla = s.layers - self.n_kda
        self.n_moe = s.layers - s.first_k_dense

    @staticmethod
    def _ffn(x: torch.Tensor, w1, w3, w2) -> torch.Tensor:
        from oracle import ops as oref

        idx = torch.zeros((x.shape[0], 1), dtype=torch.long)
        a = oref.swiglu(x, idx, w1[0][None], w1[1][None], w3[0][None], w3[1][None])[:, 0]
        return oref.dense(a, *w2)

    def seconds_per_step(self) -> tuple[float, str, int]:
        from oracle import kda_prep
        from oracle import ops as oref

        torch.set_num_threads(os.cpu_count() or 1)
        s, B = self.shape, self.batch
        scale = s.kda_head_dim ** -0.5
        t0 = time.perf_counter()
        qkv = oref.fused_qkv(self.x, *self.qkv[0], *self.qkv[1], *self.qkv[2])
        kda_prep.prepare(*qkv, *self.conv_state, *self.conv_w, self.raw_decay, self.dt_bias,
                         self.a_log, self.raw_beta, num_heads=s.kda_heads,
                         head_dim=s.kda_head_dim)
        t_qkv = time.perf_counter() - t0
        # The KDA state step's cost is linear in the batch: timed at kda_batch
        # sequences and scaled to the batch.
        st = self.state.clone()
        t0 = time.perf_counter()
        oref.kda_step(st, self.q, self.k, self.v, self.decay, self.beta, scale=scale)
        t_state = (time.perf_counter() - t0) * (B / self.kda_batch)
        t0 = time.perf_counter()
        oref.dense(self.kda_in, *self.kda_o)
        t_kda_block = t_qkv + t_state + (time.perf_counter() - t0)

        t0 = time.perf_counter()
        oref.dense(self.x, *self.mla_q)
        oref.dense(self.latent, *self.kv_b)
        oref.dense(self.attn, *self.mla_o)
        t_mla = time.perf_counter() - t0

        t0 = time.perf_counter()
        idx, w, _ = oref.router_topk(self.x, self.router, None, s.top_k,
                                     scaling=s.routed_scaling_factor)
        shared = self._ffn(self.x, *self.experts[-1])
        t_route_shared = time.perf_counter() - t0
        touched = torch.unique(idx)
        sample = touched[: self.expert_sample].tolist()
        t0 = time.perf_counter()
        for j, e in enumerate(sample):
            rows = (idx == e).any(dim=1).nonzero()[:, 0]
            self._ffn(self.x[rows], *self.experts[j])
        t_routed = (time.perf_counter() - t0) * (touched.numel() / max(1, len(sample)))
        del shared, w
        t_moe = t_route_shared + t_routed

        t0 = time.perf_counter()
        self._ffn(self.x, *self.dense)
        t_dense = time.perf_counter() - t0
        t0 = time.perf_counter()
        oref.dense(self.x, *self.lm_head)
        t_head = (time.perf_counter() - t0) * self.LM_HEAD_FRACTION

        total = (self.n_kda * t_kda_block + self.n_mla * t_mla + self.n_moe * t_moe + t_dense
                 + t_head)
        desc = (f"oracle (torch CPU, {torch.get_num_threads()} threads) at batch {B}: one KDA "
                f"block (q/k/v, preparation, state step at {self.kda_batch} sequences scaled x"
                f"{B / self.kda_batch:g}, o_proj), one MLA block (q_proj, kv_b, o_proj), one "
                f"MoE layer (router, shared expert, {len(sample)} of the {touched.numel()} "
                f"touched routed experts scaled to all), the layer-0 dense MLP and "
                f"1/{self.LM_HEAD_FRACTION} of the lm_head rows; per-step time extrapolated to "
                f"{self.n_kda} KDA + {self.n_mla} MLA blocks, {self.n_moe} MoE layers, layer 0 "
                f"and the full lm_head")
        return total, desc, torch.get_num_threads()


def cpu_median(sampler, warmup: int = 3, runs: int = 10) -> tuple[float, str, int, int]:
    """Median seconds per step of ``sampler`` after ``warmup`` untimed samples."""
    for _ in range(warmup):
        sampler.seconds_per_step()
    times, desc, cores = [], "", 1
    for _ in range(runs):
        t, desc, cores = sampler.seconds_per_step()
        times.append(t)
    return statistics.median(times), desc, cores, runs


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


def _capture(fn, x):
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(x)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn(x)
    torch.cuda.synchronize()
    return g, out


def _time_graph(g, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        g.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3 / steps


def _time_launches(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / 1e3 / steps


def _max_over_ranks(value: float, dist) -> float:
    """The largest of every rank's value (every rank gets it); NCCL groups
    reduce on the GPU, others (gloo) on the CPU."""
    if dist is None:
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _profile_traffic_ratio() -> tuple[float | None, str | None]:
    """DRAM traffic over algorithmic bytes of step_kernel from the committed ncu
    summary (profiles/step_kernel_traffic.txt: 'key value' lines)."""
    path = ROOT / "profiles" / "step_kernel_traffic.txt"
    try:
        vals = {}
        for line in path.read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and not line.startswith("#"):
                vals[parts[0]] = float(parts[1])
        return vals["dram_bytes"] / vals["algorithmic_bytes"], str(path.relative_to(ROOT))
    except Exception:
        return None, None


def _timed(step_fn, steps: int, warmup: int, dist, local_rank: int) -> tuple[float, dict]:
    """Seconds per step (device time, max over ranks) of ``steps`` calls after
    ``warmup`` untimed ones, barrier and synchronize on both sides; the SM
    clocks are sampled during the timed region."""
    if dist is not None:
        dist.barrier()
    for _ in range(max(warmup, 3)):
        step_fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            step_fn()
        end.record()
        torch.cuda.synchronize()
    step_s = _max_over_ranks(start.elapsed_time(end) / 1e3 / steps, dist)
    if dist is not None:
        dist.barrier()
    return step_s, clocks.summary()


def _e2e(step_fn, static_x: torch.Tensor, x_host: torch.Tensor, out_buf: torch.Tensor,
         steps: int, dist) -> tuple[float, int, int]:
    """The step through the public API with the input copied host->device and
    the logits device->host (pinned buffers) every step."""
    host_x = torch.empty(static_x.shape, dtype=static_x.dtype, pin_memory=True)
    host_x.copy_(x_host)
    host_out = torch.empty(out_buf.shape, dtype=out_buf.dtype, pin_memory=True)

    def e2e_step():
        static_x.copy_(host_x, non_blocking=True)
        step_fn()
        host_out.copy_(out_buf, non_blocking=True)

    if dist is not None:
        dist.barrier()
    e2e_s = _max_over_ranks(_time_launches(e2e_step, max(1, steps), 2), dist)
    return (e2e_s, host_x.numel() * host_x.element_size(),
            host_out.numel() * host_out.element_size())


def _capture_all(fn, x, dist):
    """Capture fn(x) in a CUDA graph on every rank, the NCCL exchanges of the
    expert-parallel layers included (their sizes are fixed, and nothing in the
    step reads device data on the host).  The ranks agree on the outcome with
    an all-reduce of their success flags, so either every rank replays its
    graph or every rank runs eager launches: all of them always take the same
    collective steps."""
    graph, out, ok = None, None, 1
    try:
        graph, out = _capture(fn, x)
    except Exception as exc:  # noqa: BLE001 - any capture failure falls back to eager
        print(f"[bench] graph capture failed: {type(exc).__name__}: {exc}", file=sys.stderr)
        graph, out, ok = None, None, 0
        torch.cuda.synchronize()
    if dist is not None:
        flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item())
    if not ok:
        graph, out = None, None
    return graph, out


def _recurrent_states(model) -> list[torch.Tensor]:
    """The tensors a decode step updates in place: KDA and convolution states."""
    out = []
    for lw in model.layers:
        if lw.kda_state is not None:
            out.append(lw.kda_state)
        if lw.conv_state is not None:
            out.extend(lw.conv_state)
    return out


def _graph_parity(model, graph, graph_out, static_x, dist) -> tuple[bool, float]:
    """One graph replay against one eager step from the same states (restored
    in between and afterwards): every rank's logits must match its eager
    step's, within the tolerance of the batch-1 comparison.  The ranks agree
    on the outcome.  Returns (ok on every rank, this rank's largest |diff|)."""
    states = _recurrent_states(model)
    saved = [t.clone() for t in states]
    graph.replay()
    torch.cuda.synchronize()
    ref = graph_out.float().clone()
    for t, v in zip(states, saved):
        t.copy_(v)
    eager = model.step(static_x).float()
    torch.cuda.synchronize()
    for t, v in zip(states, saved):
        t.copy_(v)
    diff = (eager - ref).abs()
    tol = torch.maximum(torch.full_like(ref, 1e-3), 2e-2 * ref.abs())
    ok = int(bool((diff <= tol).all().item()))
    worst = float(diff.max().item())
    if dist is not None:
        flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item())
    return bool(ok), worst


def _ep_step_bytes(model) -> dict[str, int]:
    """Algorithmic bytes of one expert-parallel step on this rank: every dense
    matrix and the lm_head once, the routers, the local experts the step
    touched (plus the shared expert) per MoE layer, the KDA states read and
    written, activations in and out."""
    out = model.step_bytes([1] * sum(1 for lw in model.layers if lw.moe is not None))
    expert_bytes = 0
    for li, ep in (model.ep_layers or {}).items():
        b = ep.bank
        per_expert = sum(t[0].numel() * t.element_size() for t in (
            b.w1_packed, b.w1_scales, b.w2_packed, b.w2_scales, b.w3_packed, b.w3_scales))
        expert_bytes += per_expert * (ep.touched_local_experts() + 1)
    out["total"] += expert_bytes - out["experts"]
    out["experts"] = expert_bytes
    return out


def _ep_launches(model) -> int:
    """This library's kernel launches in one expert-parallel step (the NCCL
    exchanges and torch's small copies not counted)."""
    from local_kimi_b200 import ops

    s, b = model.shape, model.batch
    tc = lambda n, k: ops.prefer_tc(b, n, k, model.group)  # noqa: E731
    proj = s.kda_heads * s.kda_head_dim
    n = 1  # lm_head
    for lw in model.layers:
        if lw.kind == "kda":
            n += 3   # q/k/v (one launch on either path), preparation + KDA step, o_proj
        else:
            both = tc(s.mla_heads * s.mla_q_head_dim, s.hidden) and tc(
                s.mla_heads * s.mla_kv_head_dim, s.kv_lora_rank)
            n += (2 if both else 1) + 1
        # MoE: router, dispatch, expert gate/up and down (the shared expert's
        # rows ride in the same two launches), combine.
        n += 2 if lw.dense_mlp is not None else 5
    return n


def _roofline(nbytes: int, step_s: float, kernel: str, traffic=None, traffic_source=None):
    peak, peak_src = _peak_hbm()
    achieved = nbytes / step_s / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "traffic_source": traffic_source, "kernel": kernel, "peak_source": peak_src,
            "bytes_per_launch": nbytes}


def _bs1_record(base, args, with_cpu: bool) -> dict:
    """Batch 1 on the decode-step executor (the whole step in one persistent
    launch), the same step as per-operation launches in a CUDA graph beside it,
    the two paths' logits compared; roofline against the measured HBM peak."""
    model = base.with_batch(1, seed=0)
    model.kda_prepare = False      # the executor's programs take fixed KDA inputs
    counts = model.touched_experts(model.x0)
    nbytes = model.step_bytes(counts)
    static_x = model.x0.clone()
    graph, graph_out = _capture(model.step, static_x)
    per_op_s = _time_graph(graph, max(10, args.steps // 2), 3)
    prog, buf = model.build_program(static_x)
    out_buf = buf["logits"]
    kda = [lw for lw in model.layers if lw.kda_state is not None]
    states = [lw.kda_state.clone() for lw in kda]
    graph.replay()
    torch.cuda.synchronize()
    ref = graph_out.float().clone()
    for lw, st in zip(kda, states):
        lw.kda_state.copy_(st)
    prog.launch()
    torch.cuda.synchronize()
    diff = (out_buf.float() - ref).abs()
    tol = torch.maximum(torch.full_like(ref, 1e-3), 2e-2 * ref.abs())
    parity = float((diff <= tol).float().mean().item())
    del graph
    step_s, clocks = _timed(prog.launch, args.steps, args.warmup, None, 0)
    e2e_s, h2d, d2h = _e2e(prog.launch, static_x, model.x0.cpu(), out_buf, args.steps, None)
    ratio, src = _profile_traffic_ratio()
    rec = {
        "workload": ("C4 hot-path decode step at batch 1 on the decode-step executor (KDA "
                     "inputs fixed: the preparation is not part of the executor's programs)"),
        "value": round(1 / step_s, 2), "unit": "tok/s", "ms_per_step": round(step_s * 1e3, 4),
        "e2e": {"value": round(1 / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": _roofline(nbytes["total"], step_s,
                              "step_kernel (the whole step in one launch)",
                              int(nbytes["total"] * ratio) if ratio else None,
                              f"ncu dram bytes / algorithmic bytes of {src}, times this "
                              f"step's algorithmic bytes" if ratio else None),
        "per_op_graph": {"ms_per_step": round(per_op_s * 1e3, 4),
                         "value": round(1 / per_op_s, 2),
                         "launches_per_step": model.launches_per_step},
        "parity_vs_per_op": round(parity, 6), "launches_per_step": 1,
        "gpu_launches": args.steps, "step_bytes": nbytes, "clocks": clocks,
    }
    if with_cpu:
        cpu_s, desc, cores = CpuSample(1, args.group, model).seconds_per_step()
        rec["cpu_baseline"] = {"value": round(1 / cpu_s, 4), "unit": "tok/s", "cores": cores,
                               "kind": "port", "sample": desc + " (one sample)"}
    return rec


def _batch_record(base, batch: int, args) -> dict:
    """A batch of ``batch`` tokens through the per-operation path (registry
    ops: the projection engine for few tokens, the tcgen05 tensor-core path for
    many) captured in one CUDA graph."""
    model = base.with_batch(batch, seed=batch)
    counts = model.touched_experts(model.x0)
    nbytes = model.step_bytes(counts)
    static_x = model.x0.clone()
    graph, out_buf = _capture(model.step, static_x)
    step_s, clocks = _timed(graph.replay, args.steps, args.warmup, None, 0)
    e2e_s, h2d, d2h = _e2e(graph.replay, static_x, model.x0.cpu(), out_buf, args.steps, None)
    del graph
    return {
        "workload": f"C4 hot-path decode step at batch {batch}, per-operation CUDA graph",
        "value": round(batch / step_s, 2), "unit": "tok/s",
        "ms_per_step": round(step_s * 1e3, 4),
        "e2e": {"value": round(batch / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": _roofline(nbytes["total"], step_s, "all launches of the step"),
        "launches_per_step": model.launches_per_step, "step_bytes": nbytes, "clocks": clocks,
    }


def _moe_layers_record(base, args) -> dict:
    """Configs C1 (1 token) and C3 (64 tokens, expert popularity skewed
    ~Zipf(1.1) by the router bias of a seeded expert permutation): the MoE
    layer (router -> gate/up + SwiGLU -> down + combine) of every MoE layer of
    the model back to back in one CUDA graph; bytes = router + the touched
    experts' three matrices."""
    import copy

    from local_kimi_b200.moe import moe_forward

    peak, _ = _peak_hbm()
    moes = [lw.moe for lw in base.layers if lw.moe is not None]
    experts = moes[0].num_experts
    per_expert = sum(t[0].numel() * t.element_size() for t in (
        moes[0].w1_packed, moes[0].w1_scales, moes[0].w2_packed, moes[0].w2_scales,
        moes[0].w3_packed, moes[0].w3_scales))
    router_bytes = moes[0].router_weight.numel() * 2
    out = {}
    for name, tokens, zipf in (("C1", 1, 0.0), ("C3", 64, 1.1)):
        layers = moes
        if zipf > 0:
            g = torch.Generator().manual_seed(7)
            perm = torch.randperm(experts, generator=g)
            bias = torch.empty(experts)
            bias[perm] = 0.25 * torch.arange(1, experts + 1, dtype=torch.float32).pow(-zipf)
            layers = []
            for m in moes:
                mm = copy.copy(m)
                mm.router_bias = bias.to(m.router_weight.device)
                layers.append(mm)
        gx = torch.Generator(device="cuda")
        gx.manual_seed(5 + tokens)
        x = torch.randn((tokens, base.shape.hidden), generator=gx, device="cuda").to(
            torch.bfloat16)
        touched, loads = [], []
        for m in layers:
            _, idx, _ = moe_forward(x, m)
            cnt = torch.bincount(idx.reshape(-1), minlength=experts)
            loads.append(int(cnt.max()))
            touched.append(int((cnt > 0).sum()) + 1)
        nbytes = sum(t * per_expert + router_bytes for t in touched)
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for m in layers:
                moe_forward(x, m)
            with torch.cuda.graph(graph, stream=side):
                for m in layers:
                    moe_forward(x, m)
        torch.cuda.current_stream().wait_stream(side)
        t = _time_graph(graph, max(5, args.steps), 3)
        del graph
        gbs = nbytes / t / 1e9
        out[name] = {"tokens": tokens, "zipf": zipf, "layers": len(layers),
                     "us_per_layer": round(t * 1e6 / len(layers), 2),
                     "touched_experts_mean": round(sum(touched) / len(touched), 1),
                     "max_tokens_per_expert": max(loads),
                     "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}
    out["timing"] = "CUDA graph of the model's MoE layers back to back, replayed"
    return out


def _sweep_record(args) -> dict:
    """The C2 dense sweep at M 1, 16 and 64 through the registry op (engine or
    tensor-core path by shape): time, HBM GB/s and fraction of the peak."""
    from local_kimi_b200 import ops

    peak, _ = _peak_hbm()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    points = []
    for name, k, n in (("qkv", 2304, 12288), ("o_proj", 4096, 2304),
                       ("shared_gate_up", 2304, 2048), ("lm_head", 2304, 163840)):
        w = (0.02 * torch.randn((n, k), generator=gen, device="cuda")).to(torch.bfloat16)
        packed, scales = ops.quantise(w, args.group)
        del w
        wbytes = packed.numel() + scales.numel() * 2
        copies = [(packed.clone(), scales.clone())
                  for _ in range(max(1, -(-400 * 2**20 // wbytes)))]
        for m in (1, 16, 64):
            x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
            t = _time_copies(ops.w4a16_dense, x, copies, 3)
            gbs = (wbytes + 2 * m * k + 2 * m * n) / t / 1e9
            path = "tc" if ops.prefer_tc(m, n, k, args.group) else "engine"
            points.append({"shape": name, "M": m, "path": path, "us": round(t * 1e6, 2),
                           "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)})
        del copies, packed, scales
        torch.cuda.empty_cache()
    return {"timing": "CUDA-graph replay over weight copies > 400 MB", "points": points}


WORKLOAD = ("C5 batch decode: {total} concurrent sequences in total ({per} per rank), the "
            "Kimi-Linear-48B-A3B W4A16 hot-path decode step ({layers} layers: INT4 attention "
            "projections, KDA decode preparation (short convolutions, gates, q/k "
            "normalisation), KDA state step, MoE router + experts + combine, INT4 lm_head) "
            "with every MoE layer expert-parallel over the {world} rank(s) ({experts} routed "
            "experts per rank, fixed-capacity exchange, NCCL all-to-all over NVLink); norms, "
            "MLA softmax attention and the BF16 projections (incl. the gate inputs) not "
            "computed")


def _progress(rank: int, what: str) -> None:
    """One line per phase on stderr, so that a stalled run shows where it stopped."""
    print(f"[bench] rank {rank} {time.strftime('%H:%M:%S')} {what}", file=sys.stderr,
          flush=True)


def run_b200(args, rank: int, world: int, local_rank: int) -> dict | None:
    import __graft_entry__ as entry

    entry.build()
    from local_kimi_b200 import _lib
    from local_kimi_b200.decode import HotPathDecoder

    torch.cuda.set_device(local_rank)
    dist = None
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
        group = dist.group.WORLD
    _lib.set_pdl(not args.no_pdl)
    if args.total_batch % world:
        raise SystemExit("--total-batch must divide over the ranks")
    per = args.total_batch // world

    _progress(rank, f"process group ready ({world} rank(s)); building weights")
    base = HotPathDecoder(1, group=args.group, layers=args.layers, seed=0)
    # Each rank's own sequences (the weights are the same on every rank).
    model = base.with_batch(per, seed=100 + rank)
    records = {}
    if world == 1 and not args.headline_only:
        records["bs1"] = _bs1_record(base, args, with_cpu=False)
        records["bs32"] = _batch_record(base, 32, args)
        if not args.no_sweep:
            records["dense_sweep"] = _sweep_record(args)
            records["moe_layers"] = _moe_layers_record(base, args)
    _progress(rank, "weights built; sub-records done; sharding experts")
    model.enable_expert_parallel(group)
    static_x = model.x0.clone()
    model.step(static_x)                         # routing for the byte count
    _progress(rank, "first expert-parallel step done")
    torch.cuda.synchronize()
    nbytes = _ep_step_bytes(model)
    graph, graph_out = _capture_all(model.step, static_x, dist)
    graph_check = None
    if graph is not None:
        # The replayed graph (at N > 1 with its exchanges) gives an eager step's logits.
        ok, worst = _graph_parity(model, graph, graph_out, static_x, dist)
        graph_check = {"graph_vs_eager_max_abs_diff": worst, "agreed": ok}
        if not ok:
            print(f"[bench] rank {rank}: graph logits differ from eager (max {worst})",
                  file=sys.stderr)
            graph, graph_out = None, None
    if graph is not None:
        step_fn, out_buf, launch = graph.replay, graph_out, "one CUDA graph per step"
    else:
        holder = {}

        def step_fn():
            holder["out"] = model.step(static_x)

        step_fn()
        torch.cuda.synchronize()
        out_buf, launch = holder["out"], "eager launches (graph capture unavailable)"
    _progress(rank, f"timing ({launch})")
    step_s, clocks = _timed(step_fn, args.steps, args.warmup, dist, local_rank)
    e2e_s, h2d, d2h = _e2e(step_fn, static_x, model.x0.cpu(), out_buf, args.steps, dist)
    _progress(rank, "timed")

    if args.profile_step:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        model.step(static_x)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.headline_only):
        cpu_s, desc, cores, runs = cpu_median(BatchCpuSample(per, args.group))
        cpu = {"value": round(per / cpu_s, 4), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": desc + f"; median of {runs} samples after 3 warm-ups",
               "seconds_per_step": round(cpu_s, 3)}
    per_layer_launches = 9                        # router, dispatch, 2 exchanges, 2+2 expert, combine
    out = {
        "metric": METRIC,
        "value": round(args.total_batch / step_s, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights of the real shapes, seeded; per-rank tokens)",
        "config": {
            "workload": WORKLOAD.format(total=args.total_batch, per=per, world=world,
                                        experts=256 // world, layers=model.nlayers),
            "total_batch": args.total_batch, "batch_per_rank": per,
            "group_size": args.group, "layers": model.nlayers,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "launch": launch,
            "graph_check": graph_check,
            "l2": "inputs larger than L2 (each step streams GBs of weights and KDA state)",
        },
        "e2e": {"value": round(args.total_batch / e2e_s, 2), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": _roofline(nbytes["total"], step_s,
                              "all launches of the step (rank 0's bytes)"),
        "gpu_launches": _ep_launches(model) * args.steps,
        "launches_per_step": _ep_launches(model),
        "step_bytes": nbytes,
        "clocks": clocks,
    }
    if cpu is not None:
        out["cpu_baseline"] = cpu
    out.update(records)
    if dist is not None:
        # Every reference to a graph that holds NCCL kernels goes before the
        # process group (the bound replay method keeps the graph alive).
        torch.cuda.synchronize()
        step_fn = None
        del graph, step_fn
        gc.collect()
        dist.destroy_process_group()
    return out if rank == 0 else None


def run_reference(args, rank: int, world: int, local_rank: int) -> dict | None:
    """The reference path restated in oracle/ on the host cores (rank 0 only),
    on the b200 arm's workload: each step a bounded sample of the batch decode
    step (BatchCpuSample), extrapolated."""
    if rank != 0:
        return None
    sample = BatchCpuSample(args.total_batch, args.group)
    warm = max(args.warmup, 3)
    steps = max(1, args.steps)
    step_s, desc, cores, _ = cpu_median(sample, warmup=warm, runs=steps)
    value = round(args.total_batch / step_s, 4)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights of the real shapes, seeded)",
        "config": {"workload": WORKLOAD.format(total=args.total_batch, per=args.total_batch,
                                               world=1, experts=256, layers=27) + " (CPU sample)",
                   "total_batch": args.total_batch, "group_size": args.group},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": desc + f"; median of {steps} samples after {warm} warm-ups"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def _peak_tflops() -> tuple[float, str]:
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(data["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def _time_copies(fn, x, copies, warmup: int) -> float:
    """Seconds per call of fn(x, packed, scales), replayed as one CUDA graph over
    weight copies larger than L2."""
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for pk, sc in copies:
            fn(x, pk, sc)
        with torch.cuda.graph(graph, stream=side):
            for pk, sc in copies:
                fn(x, pk, sc)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(max(warmup, 3)):
        graph.replay()
    reps = max(2, 60 // len(copies))
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    del graph
    return start.elapsed_time(end) / 1e3 / (reps * len(copies))


def run_dense_sweep(args) -> dict:
    """The dense W4A16 sweep: y[M,N] = x[M,K] . dequant(W)^T for the decode
    shapes, group args.group.  The projection engine (path "gemv") at M in
    {1, 4, 16, 64} and the tcgen05 tensor-core path (path "tc") at M in
    {16, 32, 64, 128, 256}.  Each point replays a CUDA graph of calls over
    enough weight copies to exceed 400 MB (inputs larger than L2, no host
    launch gaps); bytes = packed weights + scales + activations + outputs;
    the tc points also give the tensor-pipe fraction (2 M N K flops over the
    measured bf16 peak)."""
    from local_kimi_b200 import ops

    peak, peak_src = _peak_hbm()
    tpeak, tpeak_src = _peak_tflops()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    shapes = [("qkv", 2304, 12288), ("o_proj", 4096, 2304), ("shared_gate_up", 2304, 2048),
              ("lm_head", 2304, 163840)]
    gemv_ms, tc_ms = (1, 4, 16, 64), (16, 32, 64, 128, 256)
    if args.wide_sweep:
        shapes += [("mla_q", 2304, 6144), ("mla_kv_b", 512, 8192), ("dense_up", 2304, 9216),
                   ("dense_down", 9216, 2304)]
        gemv_ms, tc_ms = (1, 4, 16, 32, 64, 128, 256), (16, 32, 64, 128, 256)
    paths = [("gemv", ops.w4a16_dense, gemv_ms), ("tc", ops.w4a16_dense_tc, tc_ms)]
    points = []
    for name, k, n in shapes:
        w = (0.02 * torch.randn((n, k), generator=gen, device="cuda")).to(torch.bfloat16)
        packed, scales = ops.quantise(w, args.group)
        del w
        wbytes = packed.numel() + scales.numel() * 2
        copies = [(packed.clone(), scales.clone())
                  for _ in range(max(1, -(-400 * 2**20 // wbytes)))]
        for path, fn, ms in paths:
            for m in ms:
                gen_x = torch.Generator(device="cuda")
                gen_x.manual_seed(1)
                x = torch.randn((m, k), generator=gen_x, device="cuda").to(torch.bfloat16)
                t = _time_copies(fn, x, copies, args.warmup)
                nbytes = wbytes + 2 * m * k + 2 * m * n
                gbs = nbytes / t / 1e9
                pt = {"shape": name, "K": k, "N": n, "M": m, "path": path,
                      "us": round(t * 1e6, 2), "gbs": round(gbs, 1),
                      "frac_of_peak": round(gbs / peak, 4)}
                if path == "tc":
                    pt["tensor_frac"] = round(2.0 * m * n * k / t / 1e12 / tpeak, 4)
                points.append(pt)
        del copies, packed, scales
        torch.cuda.empty_cache()
    return {"case": "dense_sweep", "group_size": args.group, "peak_gbs": peak,
            "peak_source": peak_src, "peak_bf16_tflops": tpeak, "tflops_source": tpeak_src,
            "timing": "CUDA-graph replay over weight copies > 400 MB", "points": points}


def run_moe_layers(args) -> dict:
    """Configs C1 (--batch 1) and C3 (--batch 64 --zipf 1.1): the MoE layer
    (router top-8 -> gate/up + SwiGLU over the routed and shared experts ->
    down projection + weighted combine, three launches) of the distinct MoE
    layers of a --layers model (weights > L2), captured in one CUDA graph and
    replayed; bytes = router weights + the touched experts' three matrices.
    With --zipf S the router bias of expert perm[j] is 0.25 (j+1)^-S (seeded
    permutation), which skews the choices; the realised per-expert loads are
    reported."""
    from local_kimi_b200.decode import HotPathDecoder
    from local_kimi_b200.moe import moe_forward

    peak, peak_src = _peak_hbm()
    model = HotPathDecoder(args.batch, group=args.group, layers=args.layers or 9)
    moes = [lw.moe for lw in model.layers if lw.moe is not None]
    experts = moes[0].num_experts
    if args.zipf > 0:
        g = torch.Generator().manual_seed(7)
        perm = torch.randperm(experts, generator=g)
        bias = torch.empty(experts)
        bias[perm] = 0.25 * torch.arange(1, experts + 1, dtype=torch.float32).pow(-args.zipf)
        for m in moes:
            m.router_bias = bias.to(m.router_weight.device)
    x = model.x0
    per_matrix = [m.w1_packed[0].numel() + m.w1_scales[0].numel() * 2 for m in moes]
    per_down = [m.w2_packed[0].numel() + m.w2_scales[0].numel() * 2 for m in moes]
    touched, loads = [], []
    for m in moes:
        _, idx, _ = moe_forward(x, m)
        cnt = torch.bincount(idx.reshape(-1), minlength=experts)
        loads.append(cnt)
        touched.append(int((cnt > 0).sum()) + 1)
    nbytes = sum(t * (2 * a + b) + m.router_weight.numel() * 2
                 for t, a, b, m in zip(touched, per_matrix, per_down, moes))
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for m in moes:
            moe_forward(x, m)
        with torch.cuda.graph(graph, stream=side):
            for m in moes:
                moe_forward(x, m)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    t = start.elapsed_time(end) / 1e3 / args.steps
    load = torch.stack(loads)
    gbs = nbytes / t / 1e9
    return {"case": "moe_layers", "batch": args.batch, "group_size": args.group,
            "zipf": args.zipf, "layers": len(moes), "steps": args.steps,
            "us_per_layer": round(t * 1e6 / len(moes), 2),
            "tokens_per_s_per_layer": round(args.batch * len(moes) / t, 1),
            "touched_experts_per_layer": touched, "max_tokens_per_expert": int(load.max()),
            "bytes_per_layer": nbytes // len(moes), "gbs": round(gbs, 1),
            "frac_of_peak": round(gbs / peak, 4), "peak_gbs": peak, "peak_source": peak_src,
            "launches_per_layer": 3, "timing": "CUDA graph of all layers, replayed"}


def run_case(args) -> dict:
    """One op family at full shape, launched eagerly K times after W warm-ups
    (for profilers: every launch is a separate kernel, no graph)."""
    import __graft_entry__ as entry

    entry.build()
    if args.case == "dense_sweep":
        return run_dense_sweep(args)
    if args.case == "moe_layers":
        return run_moe_layers(args)
    from local_kimi_b200 import _lib, ops
    from local_kimi_b200.decode import HotPathDecoder, KimiLinearShape
    from local_kimi_b200.moe import moe_forward

    _lib.set_pdl(not args.no_pdl)
    s = KimiLinearShape()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    x = torch.randn((args.batch, s.hidden), generator=gen, device="cuda").to(torch.bfloat16)
    if args.case == "lm_head":
        w = (torch.randn((s.vocab_size, s.hidden), generator=gen, device="cuda") * 0.02)
        packed, scales = ops.quantise(w.to(torch.bfloat16), args.group)
        del w
        fn = lambda: ops.w4a16_dense(x, packed, scales)  # noqa: E731
        nbytes = packed.numel() + scales.numel() * 2
        per_step = 1
    elif args.case == "moe":
        model = HotPathDecoder(args.batch, group=args.group, layers=2)
        layer = model.layers[1].moe
        fn = lambda: moe_forward(x, layer)  # noqa: E731
        nbytes = None
        per_step = 3
    elif args.case == "kda":
        H, D = s.kda_heads, s.kda_head_dim
        st = 0.05 * torch.randn((args.batch, H, D, D), generator=gen, device="cuda")
        q = torch.nn.functional.normalize(
            torch.randn((args.batch, H, D), generator=gen, device="cuda"), dim=-1)
        k = torch.nn.functional.normalize(
            torch.randn((args.batch, H, D), generator=gen, device="cuda"), dim=-1)
        v = 0.2 * torch.randn((args.batch, H, D), generator=gen, device="cuda")
        dec = -(0.005 + 0.075 * torch.rand((args.batch, H, D), generator=gen, device="cuda"))
        beta = torch.sigmoid(torch.randn((args.batch, H), generator=gen, device="cuda"))
        ob = torch.empty((args.batch, H, D), dtype=torch.bfloat16, device="cuda")
        fn = lambda: ops.kda_decode_step(st, q, k, v, dec, beta, scale=D ** -0.5,  # noqa: E731
                                         out_bf16=ob)
        nbytes = 2 * st.numel() * 4 + 5 * q.numel() * 4
        per_step = 1
    elif args.case == "experts":
        E, I, top_k = s.experts, s.moe_intermediate, s.top_k
        q = lambda n, kk: ops.quantise(  # noqa: E731
            (0.02 * torch.randn((E * n, kk), generator=gen, device="cuda")).to(torch.bfloat16),
            args.group)
        w1, w3, w2 = q(I, s.hidden), q(I, s.hidden), q(s.hidden, I)
        w1p, w1s = w1[0].view(E, I, -1), w1[1].view(E, I, -1)
        w3p, w3s = w3[0].view(E, I, -1), w3[1].view(E, I, -1)
        w2p, w2s = w2[0].view(E, s.hidden, -1), w2[1].view(E, s.hidden, -1)
        rows = args.batch * top_k
        idx = torch.randint(0, E, (rows, 1), generator=gen, device="cuda")
        xr = torch.randn((rows, s.hidden), generator=gen, device="cuda").to(torch.bfloat16)

        def fn():
            act = ops.w4a16_swiglu_tc(xr, idx, w1p, w1s, w3p, w3s)
            ops.w4a16_grouped_tc(act[:, 0], idx, w2p, w2s)

        touched = int(torch.unique(idx).numel())
        per_expert = sum(t[0].numel() * t.element_size() for t in (w1p, w1s, w3p, w3s, w2p, w2s))
        nbytes = touched * per_expert
        per_step = 2
    elif args.case == "program":
        model = HotPathDecoder(args.batch, group=args.group, layers=args.layers)
        prog, _ = model.build_program(model.x0.clone())
        fn = prog.launch
        nbytes = model.step_bytes(model.touched_experts(model.x0))["total"]
        per_step = 1
    else:
        model = HotPathDecoder(args.batch, group=args.group, layers=args.layers)
        fn = lambda: model.step(x)  # noqa: E731
        nbytes = None
        per_step = model.launches_per_step
    for _ in range(max(args.warmup, 1)):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    t = start.elapsed_time(end) / 1e3 / args.steps
    out = {"case": args.case, "batch": args.batch, "group_size": args.group,
           "steps": args.steps, "warmup": args.warmup, "launches_per_iteration": per_step,
           "us_per_iteration": round(t * 1e6, 2)}
    if args.case == "eager":
        nbytes = model.step_bytes(model.touched_experts(x))["total"]
    if nbytes:
        out["bytes_per_iteration"] = nbytes
        out["gbs"] = round(nbytes / t / 1e9, 1)
    return out


def run_ep_moe(args, rank: int, world: int, local_rank: int) -> dict | None:
    """One full-size MoE layer (256 experts + shared, hidden 2304, intermediate
    1024, top-8, g128, random init, seeded) with the experts sharded over the
    ranks and --batch tokens in total (batch / world per rank, random bf16
    hidden states); K timed forwards after W warm-ups between barriers, device
    time as the max over ranks.  Every rank runs the same collectives."""
    import datetime

    import __graft_entry__ as entry
    import torch.distributed as dist

    entry.build()
    from local_kimi_b200 import ops
    from local_kimi_b200.ep import ExpertParallelMoE
    from local_kimi_b200.moe import MoELayerWeights

    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local_rank))
    E, H, I = 256, 2304, 1024
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)

    def bank(n: int, k: int):
        packed, scales = [], []
        for _ in range(E + 1):
            w = (0.02 * torch.randn((n, k), generator=gen, device="cuda")).to(torch.bfloat16)
            p, sc = ops.quantise(w, args.group)
            packed.append(p)
            scales.append(sc)
        return torch.stack(packed), torch.stack(scales)

    w1 = bank(I, H)
    w3 = bank(I, H)
    w2 = bank(H, I)
    router = (0.05 * torch.randn((E, H), generator=gen, device="cuda")).to(torch.bfloat16)
    bias = 0.01 * torch.randn((E,), generator=gen, device="cuda")
    layer = MoELayerWeights(router, bias, w1[0], w1[1], w2[0], w2[1], w3[0], w3[1])
    ep = ExpertParallelMoE(layer)
    del w1, w2, w3
    torch.cuda.empty_cache()
    if args.batch % world:
        raise SystemExit("--batch must divide over the ranks")
    per = args.batch // world
    gx = torch.Generator(device="cuda")
    gx.manual_seed(1 + rank)
    x = torch.randn((per, H), generator=gx, device="cuda").to(torch.bfloat16)
    for _ in range(max(args.warmup, 3)):
        ep.forward(x)
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        ep.forward(x)
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end) / 1e3 / args.steps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    ids = ops.payload_ids(ep.last_payload)[:, 0]
    cap = ids.numel() // world
    send = [int((ids[d * cap:(d + 1) * cap] >= 0).sum()) for d in range(world)]
    recv = [int(ep.touched_local_experts())]
    dist.destroy_process_group()
    if rank != 0:
        return None
    step_s = float(t.item())
    return {"case": "ep_moe", "metric": "MoE layer tokens/s (expert-parallel)",
            "value": round(args.batch / step_s, 1), "unit": "tok/s", "n_gpus": world,
            "ms_per_step": round(step_s * 1e3, 4), "steps": args.steps,
            "warmup": args.warmup, "scaling": "strong",
            "config": {"tokens": args.batch, "tokens_per_rank": per, "experts": E,
                       "experts_per_rank": E // world, "hidden": H, "intermediate": I,
                       "top_k": 8, "group_size": args.group,
                       "rank0_rows_sent_per_dest": send,
                       "rank0_local_experts_touched": recv[0],
                       "data": "synthetic (random-init weights and hidden states, seeded)"}}


def main() -> None:
    args = _args()
    rank, world, local_rank = _dist_env()
    if args.case == "ep_moe":
        out = run_ep_moe(args, rank, world, local_rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    if args.case != "step":
        if rank == 0:
            print(json.dumps(run_case(args)), flush=True)
        return
    if args.impl == "reference":
        out = run_reference(args, rank, world, local_rank)
    else:
        out = run_b200(args, rank, world, local_rank)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
