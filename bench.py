"""Benchmark of the B200 attention backend (one JSON line on rank 0).

Default workload (``--workload c5``): BASELINE configs[4], Gemma-3-270M-shaped
decode, batch 256 sequences per GPU, 4 query heads / 1 kv head, head_dim 256,
fp16 KV cache, context lengths ~ U[1024, 32768].  One step = one decode token
per sequence through one sliding-window-512 local layer (RoPE theta 1e4) and
one global layer (theta 1e6), each with per-head zero-centred RMS QK-norm,
i.e. two ``b2a_decode`` calls on two separate caches.  ``value`` is decode
tokens/s over all ranks (weak scaling: every rank owns its own 256 sequences,
no collective in the timed region).  ``e2e`` is the same step through the C ABI
with the step's inputs (new q/k/v, context lengths) copied from pinned host
memory and the outputs copied back inside the timed region; the KV caches are
device-resident state, as in the reference's GPU-resident decode.

Other workloads: c1 (SmolLM2 prefill, fp32), c2 (MiniLM encoder, fp16),
c3 (Qwen2.5 decode, fp16 cache), c4 (Phi-3 prefill, bf16).  At N=1 rank 0 also
times c1-c4 once and reports them under ``suite``.

``--impl reference`` times the CPU restatement of the reference's Java CPU
attention (the oracle, OpenMP over all host threads) on a bounded sample of
the same workload; the reference itself (Java 21) cannot run on this machine.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "win-directml-java_b200"))
sys.path.insert(0, REPO)

MEASURED_PEAKS = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0

WORKLOADS = {
    "c1": "SmolLM2-135M causal prefill B1 S256 9/3 D64 fp32 (configs[0])",
    "c2": "MiniLM-L6 encoder B64 S128 H12 D32 fp16 key-padding (configs[1])",
    "c3": "Qwen2.5-0.5B decode B64 14/2 D64 fp16 KV ctx~U[512,8192] (configs[2])",
    "c4": "Phi-3-mini causal prefill B8 S4096 H32 D96 bf16 (configs[3])",
    "c5": "Gemma-3-270M decode B256 4/1 D256 local W512 + global, QK-norm, fp16 KV ctx~U[1024,32768] (configs[4])",
    "c3blk": "Qwen2.5-0.5B decode attention block B64 hidden 896 14/2 D64 fp16: QKV GEMM + bias, decode, "
             "O GEMM + residual (configs[2] with its projections)",
}


def peaks():
    try:
        with open(MEASURED_PEAKS) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


# ------------------------------------------------------------------ clocks
class NvmlClockSampler:
    """Reads SM clock and clock-event reasons through NVML every 5 ms in a thread
    (read-only queries; nothing is changed on the GPU)."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpu_index: int):
        import threading
        self.gpu, self.samples, self.reasons = gpu_index, [], set()
        self.stop = threading.Event()
        self.thread = None
        self.max_mhz = None
        self.ok = False

    def _run(self, nv, h):
        while not self.stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self.stop.wait(0.005)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            idx = self.gpu
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                try:
                    idx = int(vis.split(",")[self.gpu])
                except (ValueError, IndexError):
                    pass
            h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, args=(nv, h), daemon=True)
            self.thread.start()
            self.ok = True
        except Exception:
            self.ok = False
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.ok or not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons), "source": "nvml 5 ms"}


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"b2a_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------ workloads
DECODE_SHAPES = {  # B per GPU, Hq, Hkv, D, context range, layers (window, RoPE theta)
    "c5": dict(B=256, Hq=4, Hkv=1, D=256, lo=1024, hi=32768, layers=[(512, 1e4), (0, 1e6)]),
    "c3": dict(B=64, Hq=14, Hkv=2, D=64, lo=512, hi=8192, layers=[(0, 1e6)]),
}


def decode_config(name: str, B: int, lens, max_seq: int) -> dict:
    """The `config` object of a decode workload's JSON line (both arms print the same one)."""
    sh = DECODE_SHAPES[name]
    cache_gb = len(sh["layers"]) * 2 * B * max_seq * sh["Hkv"] * sh["D"] * 2 / 1e9
    return {"workload": WORKLOADS[name], "batch_per_gpu": B, "q_heads": sh["Hq"], "kv_heads": sh["Hkv"],
            "head_dim": sh["D"], "ctx_len": f"U[{sh['lo']},{sh['hi']}]", "mean_ctx": float(np.mean(lens)),
            "layers_per_step": [("local W%d" % w) if w else "global" for w, _ in sh["layers"]],
            "kv_dtype": "f16", "l2": "inputs larger than L2 (KV caches %.1f GB)" % cache_gb}


class DecodeWorkload:
    """configs[4] (c5) or configs[2] (c3): one decode token for every sequence."""

    def __init__(self, name: str, seed: int, batch: int = 0, world: int = 1, rank: int = 0, n_layers: int = 1):
        import torch
        import b200attn
        self.torch, self.b2a, self.name = torch, b200attn, name
        if name == "c5":
            self.B, self.Hq, self.Hkv, self.D, self.lo, self.hi = 256, 4, 1, 256, 1024, 32768
            self.layers = [dict(window=512, theta=1e4), dict(window=0, theta=1e6)]
            self.layout, self.rope, self.norm = b200attn.KV_POS_MAJOR, b200attn.ROPE_GEMMA, True
        else:
            self.B, self.Hq, self.Hkv, self.D, self.lo, self.hi = 64, 14, 2, 64, 512, 8192
            # n_layers > 1: a model step, every layer with its own cache (the same sequences)
            self.layers = [dict(window=0, theta=1e6) for _ in range(n_layers)]
            self.layout, self.rope, self.norm = b200attn.KV_HEAD_MAJOR, b200attn.ROPE_NEOX, False
        if batch > 0:  # smaller batch for profiler captures only
            self.B = batch
        from b200attn import synthetic
        # One global batch of world * B sequences.  The partition unit is (sequence, kv head):
        # each rank takes a cost-balanced, equal-count shard of the units (plan_shards; cost =
        # keys attended) and runs them as sequences with one kv head and Hq/Hkv q heads.  With
        # one kv head (c5) a unit is a sequence.  The outputs are reassembled in the e2e arm.
        self.world, self.rank = world, rank
        self.seqs_per_rank = self.B
        self.Hkv_model, self.Hq_model = self.Hkv, self.Hq
        lens_all = synthetic.uniform_int(seed, self.B * world, self.lo, self.hi)
        self.plan = None
        if world > 1:
            from b200attn import sharding
            unit_lens = np.repeat(lens_all, self.Hkv)  # unit u = (sequence u // Hkv, kv head u % Hkv)
            self.plan = sharding.plan_shards(unit_lens.astype(np.int64) + 1, world)
            self.lens = np.ascontiguousarray(unit_lens[self.plan[rank]])
            self.B, self.Hq, self.Hkv = len(self.lens), self.Hq // self.Hkv, 1
        else:
            self.lens = lens_all
        self.max_seq = self.hi + 1
        g = torch.Generator(device="cuda").manual_seed(seed + rank)
        B, Hq, Hkv, D, S = self.B, self.Hq, self.Hkv, self.D, self.max_seq
        shape = (B, Hkv, S, D) if self.layout == b200attn.KV_HEAD_MAJOR else (B, S, Hkv, D)
        self.caches = []
        for _ in self.layers:
            kc = torch.empty(shape, dtype=torch.float16, device="cuda")
            vc = torch.empty(shape, dtype=torch.float16, device="cuda")
            for t in (kc, vc):
                for b in range(B):  # per-sequence slices keep the fp32 temporaries small
                    t[b].normal_(generator=g)
            self.caches.append((kc, vc))
        mk = lambda *s: torch.randn(*s, generator=g, device="cuda").to(torch.float16)
        self.q = [mk(B, Hq, D) for _ in self.layers]
        self.kn = [mk(B, Hkv, D) for _ in self.layers]
        self.vn = [mk(B, Hkv, D) for _ in self.layers]
        self.qw = torch.randn(D, generator=g, device="cuda") * 0.5 if self.norm else None
        self.kw = torch.randn(D, generator=g, device="cuda") * 0.5 if self.norm else None
        self.lens_d = torch.from_numpy(self.lens).cuda()
        self.out = [torch.empty(B, Hq, D, device="cuda") for _ in self.layers]
        self.scale = 1.0 / math.sqrt(D)
        # host-side mirrors for the end-to-end arm
        pin = lambda t: t.cpu().pin_memory()
        self.h_q = [pin(t) for t in self.q]
        self.h_kn = [pin(t) for t in self.kn]
        self.h_vn = [pin(t) for t in self.vn]
        self.h_lens = pin(self.lens_d)
        self.h_out = [torch.empty(B, Hq, D).pin_memory() for _ in self.layers]
        if world > 1:  # every rank receives the whole batch's outputs of both layers; rank 0 copies them out
            from b200attn import sharding
            self.h_out_all = torch.empty(len(self.layers), B * world, Hq, D).pin_memory()
            self.reassemble = sharding.Reassembly(self.plan, torch.device("cuda", torch.cuda.current_device()))

    def tokens_per_step(self):
        return self.seqs_per_rank

    def kernel_launches_per_step(self):
        return len(self.layers)

    def algorithmic_bytes(self):
        """KV bytes each decode launch must read + new rows written + q/o/new k/v, summed over the step."""
        total = 0
        for layer in self.layers:
            L = self.lens.astype(np.int64)
            visible = np.minimum(L + 1, layer["window"]) if layer["window"] > 0 else L + 1
            kv = int(visible.sum()) * self.Hkv * self.D * 2 * 2
            small = self.B * (self.Hq + 2 * self.Hkv) * self.D * 2 + self.B * self.Hq * self.D * 4
            total += kv + small + self.B * self.Hkv * self.D * 2 * 2
        return total

    def flops(self):
        total = 0
        for layer in self.layers:
            L = self.lens.astype(np.int64)
            visible = np.minimum(L + 1, layer["window"]) if layer["window"] > 0 else L + 1
            total += int(visible.sum()) * self.Hq * self.D * 4
        return total

    def launch(self, ctx, i, stream=None):
        layer = self.layers[i]
        kc, vc = self.caches[i]
        self.b2a.decode(ctx, self.q[i], self.kn[i], self.vn[i], kc, vc, self.lens_d, self.out[i], self.scale,
                        kv_layout=self.layout, rope_mode=self.rope, rope_theta=layer["theta"],
                        window=layer["window"], q_norm_w=self.qw, k_norm_w=self.kw, norm_eps=1e-6, stream=stream)

    def step(self, ctx, stream=None):
        for i in range(len(self.layers)):
            self.launch(ctx, i, stream)

    def step_e2e(self, ctx):
        """One step through the public API with its host transfers: the step's inputs (new q/k/v
        rows, context lengths) from pinned host memory, the outputs back to pinned host memory.
        Copies run on a copy stream: layer 1's inputs arrive while layer 0 computes and layer 0's
        outputs leave while layer 1 computes.  The step ends when its last copy has landed (the
        next step's inputs depend on this step's outputs in a real decode loop)."""
        torch = self.torch
        main = torch.cuda.current_stream()
        if not hasattr(self, "copy_stream"):
            self.copy_stream = torch.cuda.Stream()
            self.ev_in = [torch.cuda.Event() for _ in self.layers]
            self.ev_out = [torch.cuda.Event() for _ in self.layers]
            self.ev_done = torch.cuda.Event()
        cs = self.copy_stream
        cs.wait_stream(main)  # the previous step (and its copies) is complete
        with torch.cuda.stream(cs):
            self.lens_d.copy_(self.h_lens, non_blocking=True)
            for i in range(len(self.layers)):
                self.q[i].copy_(self.h_q[i], non_blocking=True)
                self.kn[i].copy_(self.h_kn[i], non_blocking=True)
                self.vn[i].copy_(self.h_vn[i], non_blocking=True)
                self.ev_in[i].record(cs)
        if self.world > 1 and not hasattr(self, "gather_stream"):
            self.gather_stream = torch.cuda.Stream()
        for i in range(len(self.layers)):
            main.wait_event(self.ev_in[i])
            self.launch(ctx, i)
            self.ev_out[i].record(main)
            if self.world == 1:
                cs.wait_event(self.ev_out[i])
                with torch.cuda.stream(cs):
                    self.h_out[i].copy_(self.out[i], non_blocking=True)
            else:
                # output reassembly per layer on a side stream, so layer i's all-gather and host
                # copy overlap layer i+1's attention: one NCCL all-gather of the equal shards,
                # scattered back into unit order; rank 0, the host that consumes the reassembled
                # batch, copies it out (every rank holds the same reassembled tensor)
                gs = self.gather_stream
                gs.wait_event(self.ev_out[i])
                with torch.cuda.stream(gs):
                    full = self.reassemble(self.out[i])
                    if self.rank == 0:
                        self.h_out_all[i].copy_(full, non_blocking=True)
        if self.world > 1:
            main.wait_stream(self.gather_stream)
        else:
            self.ev_done.record(cs)
            main.wait_event(self.ev_done)

    def e2e_bytes(self):
        h2d = self.lens.nbytes + sum(t.numel() * t.element_size() for t in self.h_q + self.h_kn + self.h_vn)
        if self.world > 1:  # the reassembled batch, copied out once (rank 0)
            d2h = self.h_out_all.numel() * self.h_out_all.element_size()
        else:
            d2h = sum(t.numel() * t.element_size() for t in self.h_out)
        return h2d, d2h

    def config(self):
        cfg = decode_config(self.name, self.seqs_per_rank, self.lens, self.max_seq)
        if self.world > 1:
            cfg["partition_unit"] = "(sequence, kv head)" if self.Hkv_model > 1 else "sequence"
            cfg["units_per_rank"] = self.B
            cfg["reassembly"] = ("NCCL all_gather of equal shards per layer in the e2e arm, overlapping the next "
                                 "layer (b200attn.sharding.Reassembly); rank 0 copies the reassembled batch to host")
        return cfg


class PrefillWorkload:
    """c1 / c4: causal prefill with fused RoPE; c2: masked encoder."""

    def __init__(self, name: str, seed: int, batch: int = 0, n_layers: int = 1):
        import torch
        import b200attn
        from b200attn import synthetic
        self.torch, self.b2a, self.name = torch, b200attn, name
        g = torch.Generator(device="cuda").manual_seed(seed)
        if name == "c1":
            self.B, self.S, self.Hq, self.Hkv, self.D, self.dt, self.theta = 1, 256, 9, 3, 64, torch.float32, 1e5
        elif name == "c4":
            self.B, self.S, self.Hq, self.Hkv, self.D, self.dt, self.theta = 8, 4096, 32, 32, 96, torch.bfloat16, 1e4
        else:
            self.B, self.S, self.Hq, self.Hkv, self.D, self.dt, self.theta = 64, 128, 12, 12, 32, torch.float16, 0
            self.lens = synthetic.uniform_int(seed, self.B if batch <= 0 else batch, 16, 128)
            self.lens_d = torch.from_numpy(self.lens).cuda()
        if batch > 0:  # smaller batch for profiler captures only
            self.B = batch
        mk = lambda h: torch.randn(self.B, self.S, h, self.D, generator=g, device="cuda").to(self.dt)
        self.q, self.k, self.v = mk(self.Hq), mk(self.Hkv), mk(self.Hkv)
        self.o = torch.empty_like(self.q)
        # n_layers > 1: a model step, every layer with its own q, k, v, o (the same sequences)
        self.layer_tensors = [(self.q, self.k, self.v, self.o)]
        for _ in range(n_layers - 1):
            q, k, v = mk(self.Hq), mk(self.Hkv), mk(self.Hkv)
            self.layer_tensors.append((q, k, v, torch.empty_like(q)))
        self.scale = 1.0 / math.sqrt(self.D)

    def tokens_per_step(self):
        return self.B * self.S

    def kernel_launches_per_step(self):
        # c2: attention; c1 (fp32): attention rotating q and k itself from the context's cached table;
        # c4 (bf16): one pre-pass (rope q, k from the cached table; convert q, k, v), attention
        per_layer = 2 if self.name == "c4" else 1
        return per_layer * len(self.layer_tensors)

    def flops(self):
        """Summed over the step's layers."""
        if self.name == "c2":
            per = 4 * self.Hq * self.D * self.S * int(self.lens.astype(np.int64).sum())
        else:
            per = 4 * self.B * self.Hq * self.D * self.S * (self.S + 1) // 2
        return per * len(self.layer_tensors)

    def algorithmic_bytes(self):
        """Summed over the step's layers."""
        e = self.q.element_size()
        return e * self.B * self.S * self.D * (2 * self.Hq + 2 * self.Hkv) * len(self.layer_tensors)

    def step(self, ctx, stream=None):
        for q, k, v, o in self.layer_tensors:
            if self.name == "c2":
                self.b2a.mha(ctx, q, k, v, o, self.scale, key_lengths=self.lens_d, layout=self.b2a.SEQ_MAJOR,
                             stream=stream)
            else:
                self.b2a.prefill_causal(ctx, q, k, v, o, self.scale, rope_mode=self.b2a.ROPE_NEOX,
                                        rope_theta=self.theta, stream=stream)


class BlockWorkload:
    """c3blk: configs[2]'s decode step with the projections around it (b2a_decode_attention_block):
    x [64, 896] -> QKV GEMM (+bias) -> fused decode (RoPE, append, GQA attention) -> O GEMM
    (+residual); random weights of Qwen2.5-0.5B's shapes (no checkpoint)."""

    def __init__(self, seed: int = 3):
        import torch
        import b200attn
        from b200attn import synthetic
        self.torch, self.b2a = torch, b200attn
        self.B, self.hidden, self.Hq, self.Hkv, self.D, self.max_seq = 64, 896, 14, 2, 64, 8193
        self.lens = synthetic.uniform_int(seed, self.B, 512, 8192)
        g = torch.Generator(device="cuda").manual_seed(seed)
        nqkv = (self.Hq + 2 * self.Hkv) * self.D
        w = lambda *sh: (torch.randn(*sh, generator=g, device="cuda") / math.sqrt(sh[-1])).half()
        self.x = torch.randn(self.B, self.hidden, generator=g, device="cuda").half()
        self.res = torch.randn(self.B, self.hidden, generator=g, device="cuda").half()
        self.wqkv, self.wo = w(nqkv, self.hidden), w(self.hidden, self.Hq * self.D)
        self.bqkv = 0.1 * torch.randn(nqkv, generator=g, device="cuda")
        shape = (self.B, self.Hkv, self.max_seq, self.D)
        self.kc = torch.empty(shape, dtype=torch.float16, device="cuda")
        self.vc = torch.empty(shape, dtype=torch.float16, device="cuda")
        for t in (self.kc, self.vc):
            for b in range(self.B):
                t[b].normal_(generator=g)
        self.lens_d = torch.from_numpy(self.lens).cuda()
        self.y = torch.empty(self.B, self.hidden, dtype=torch.float16, device="cuda")

    def tokens_per_step(self):
        return self.B

    def kernel_launches_per_step(self):
        return 3

    def algorithmic_bytes(self):
        kv = int((self.lens.astype(np.int64) + 1).sum()) * self.Hkv * self.D * 2 * 2
        weights = (self.wqkv.numel() + self.wo.numel()) * 2
        act = self.B * self.hidden * 2 * 3 + self.B * self.Hkv * self.D * 2 * 2
        return kv + weights + act

    def flops(self):
        proj = 2 * self.B * self.hidden * (self.wqkv.shape[0] + self.Hq * self.D)
        return proj + int((self.lens.astype(np.int64) + 1).sum()) * self.Hq * self.D * 4

    def step(self, ctx, stream=None):
        self.b2a.decode_attention_block(ctx, self.x, self.wqkv, self.bqkv, self.kc, self.vc, self.lens_d, self.wo,
                                        self.res, self.y, num_q_heads=self.Hq, num_kv_heads=self.Hkv, scale=0.125,
                                        rope_theta=1e6, stream=stream)


def capture_graph(torch, fn):
    """CUDA graph of fn(), which launches its work on the current stream (the library
    calls take torch's current stream), or None when capture is not possible.  Replaying
    it keeps Python and ctypes call overhead out of device-timed intervals: for kernels
    of tens of microseconds a host-driven launch leaves the GPU idle between steps."""
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()  # warm on the capture's stream family: no first-use work inside the capture
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g
    except Exception as e:  # report and time direct launches instead
        print(f"# CUDA graph capture failed ({type(e).__name__}: {e}); timing direct launches", file=sys.stderr)
        torch.cuda.synchronize()
        return None


def time_steps(torch, fn, steps, flush=None):
    """Per-step CUDA-event durations (ms) on the current stream."""
    s = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        if flush is not None:
            flush()
        a.record(s)
        fn()
        b.record(s)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def run_suite(ctx, hbm, tflops, src):
    import torch
    # L2 flush between reps: write 512 MB (every line of the 126 MB L2 evicted), then read
    # 256 MB of another buffer so that the lines L2 holds when the timed launch starts are
    # clean; a write alone leaves ~126 MB of dirty lines whose write-back the timed kernel
    # would pay for (c3 reads only 130 MB)
    flush_buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    clean_buf = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    clean_sum = torch.empty((), dtype=torch.float32, device="cuda")

    def flush():
        flush_buf.fill_(1.0)
        torch.sum(clean_buf, dim=0, out=clean_sum)
    out = {}
    for name in ("c1", "c2", "c3", "c4", "c3blk"):
        w = DecodeWorkload(name, 3) if name == "c3" else BlockWorkload() if name == "c3blk" else \
            PrefillWorkload(name, {"c1": 1, "c2": 2, "c4": 4}[name])
        for _ in range(3):
            w.step(ctx)
        torch.cuda.synchronize()
        # one step as a CUDA graph, captured after this workload's warm-up (the context's
        # workspaces have their final size) and dropped before the next workload runs
        g = capture_graph(torch, lambda: w.step(ctx))
        ms = statistics.mean(time_steps(torch, (lambda: g.replay()) if g is not None else (lambda: w.step(ctx)),
                                        10, flush))
        del g
        entry = {"workload": WORKLOADS[name], "ms": round(ms, 4), "l2": "flushed (512 MB write + 256 MB read)",
                 "tokens_per_s": round(w.tokens_per_step() / (ms / 1e3), 1)}
        gbs = w.algorithmic_bytes() / (ms / 1e3) / 1e9
        tfs = w.flops() / (ms / 1e3) / 1e12
        entry["hbm_gbs"] = round(gbs, 1)
        entry["hbm_frac"] = round(gbs / hbm, 4)
        entry["tflops"] = round(tfs, 2)
        entry["tensor_frac"] = round(tfs / tflops, 4)
        entry["bound"] = "tensor" if name == "c4" else "hbm"
        entry["peak_source"] = src
        del w
        torch.cuda.empty_cache()
        if name in MODEL_LAYERS:
            entry["model_step"] = model_step_entry(ctx, torch, name, hbm, time_steps_fn=time_steps, flush=flush)
        out[name] = entry
    return out


# Layers of the model each latency-bound suite config is shaped on: SmolLM2-135M (30), MiniLM-L6 (6),
# Qwen2.5-0.5B (24).  Their attention launches run back to back in a real forward or decode step.
MODEL_LAYERS = {"c1": 30, "c2": 6, "c3": 24}


def model_step_entry(ctx, torch, name, hbm, time_steps_fn, flush):
    """The config's attention over every layer of its model in one step: each layer has its own
    tensors (caches), the layers' launches run back to back in one CUDA graph, L2 is flushed before
    each step.  Reports the time per layer, where a single launch's fixed cost (the launch and the
    first loads of every CTA) overlaps the previous layer as it does in a model."""
    L = MODEL_LAYERS[name]
    w = DecodeWorkload(name, 3, n_layers=L) if name == "c3" else \
        PrefillWorkload(name, {"c1": 1, "c2": 2}[name], n_layers=L)
    for _ in range(2):
        w.step(ctx)
    torch.cuda.synchronize()
    g = capture_graph(torch, lambda: w.step(ctx))
    ms = statistics.mean(time_steps_fn(torch, (lambda: g.replay()) if g is not None else (lambda: w.step(ctx)),
                                       5, flush))
    del g
    per = ms / L
    gbs = w.algorithmic_bytes() / L / (per / 1e3) / 1e9
    entry = {"layers": L, "ms_per_step": round(ms, 4), "ms_per_layer": round(per, 4),
             "hbm_gbs_per_layer": round(gbs, 1), "hbm_frac_per_layer": round(gbs / hbm, 4),
             "tokens_per_s": round(w.tokens_per_step() / (ms / 1e3), 1),
             "l2": "flushed before each step; every layer's tensors distinct"}
    del w
    torch.cuda.empty_cache()
    return entry


# ------------------------------------------------------------------ CPU reference arm
def host_threads() -> int:
    """Host cores this process may run on.  Passed to the oracle explicitly: torchrun sets
    OMP_NUM_THREADS=1 in its workers, which would leave the CPU arm on one thread at N > 1."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


class CpuDecodeSample:
    """A bounded sample of the c5 workload for the CPU restatement (OpenMP over all host
    threads): n_seq of the benchmark's 256 sequences, taken at the midpoints of n_seq equal
    quantile bins of their context lengths so that the sample's length mix (and mean) is the
    whole batch's, in the GPU arm's position-major cache layout; one step = one decode token
    per sampled sequence through the local W512 and the global layer."""

    def __init__(self, n_seq: int, seed: int = 5):
        import oracle
        from b200attn import synthetic
        self.oracle = oracle
        sh = DECODE_SHAPES["c5"]
        self.all_lens = synthetic.uniform_int(seed, sh["B"], sh["lo"], sh["hi"])
        self.lens = np.ascontiguousarray(self.all_lens[synthetic.stratified_sample(self.all_lens, n_seq)])
        self.n = n_seq
        self.D, self.Hq, self.Hkv = sh["D"], sh["Hq"], sh["Hkv"]
        self.max_seq = int(self.lens.max()) + 1
        rng = np.random.default_rng(seed)
        shape = (n_seq, self.max_seq, self.Hkv, self.D)  # position-major, as the GPU arm's caches
        self.caches = []
        for _ in sh["layers"]:  # one cache per layer, as on the GPU
            kc = oracle.round_to(rng.standard_normal(shape, dtype=np.float32), oracle.F16).reshape(shape)
            vc = oracle.round_to(rng.standard_normal(shape, dtype=np.float32), oracle.F16).reshape(shape)
            self.caches.append((kc, vc))
        r = lambda *s: oracle.round_to(rng.standard_normal(s, dtype=np.float32), oracle.F16).reshape(s)
        self.q, self.kn, self.vn = r(n_seq, self.Hq, self.D), r(n_seq, self.Hkv, self.D), r(n_seq, self.Hkv, self.D)
        self.w = (0.5 * rng.standard_normal(self.D)).astype(np.float32)
        self.threads = host_threads()

    def describe(self) -> str:
        return (f"{self.n} of the 256 sequences (stratified by context length: sample mean "
                f"{self.lens.mean():.0f} vs batch mean {self.all_lens.mean():.0f}), position-major fp16-valued "
                f"caches, one local W512 + one global layer per step")

    def step(self):
        o = self.oracle
        for (kc, vc), (window, theta) in zip(self.caches, DECODE_SHAPES["c5"]["layers"]):
            o.decode(self.q, self.kn, self.vn, kc, vc, self.lens, B=self.n, Hq=self.Hq, Hkv=self.Hkv, D=self.D,
                     max_seq=self.max_seq, scale=1 / 16, rope_theta=theta, rope_mode=o.ROPE_GEMMA, window=window,
                     cache_layout=o.KV_POS_MAJOR, q_norm_w=self.w, k_norm_w=self.w,
                     softmax_mode=o.SOFTMAX_GEMMA, n_threads=self.threads, inplace=True)


CPU_SAMPLE_SEQS = 16


def cpu_decode_sample(n_seq: int, max_seconds: float = 12.0):
    """Times the CPU restatement on a bounded sample; returns (tokens/s, threads, seconds, steps, sample)."""
    smp = CpuDecodeSample(n_seq)
    smp.step()  # warm caches / thread pool
    steps, t0 = 0, time.perf_counter()
    while True:
        smp.step()
        steps += 1
        el = time.perf_counter() - t0
        if el >= max_seconds or steps >= 200:
            break
    return n_seq * steps / el, smp.threads, el, steps, smp.describe()


def reference_arm(args):
    """The reference arm: the reference's CPU attention restated in C (no JDK exists here), timed on
    the host's cores on a bounded sample of the c5 workload; the same metric, unit and config as the
    GPU arm.  Under torchrun only rank 0 runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    from b200attn import synthetic
    oracle.build()
    smp = CpuDecodeSample(CPU_SAMPLE_SEQS)
    # each step is the bounded sample; keep the whole run within a few minutes
    steps = max(1, min(args.steps, 200))
    for _ in range(args.warmup):
        smp.step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        smp.step()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = smp.n / (ms / 1e3)
    threads = host_threads()
    sh = DECODE_SHAPES["c5"]
    config = dict(decode_config("c5", sh["B"], synthetic.uniform_int(5, sh["B"] * args.gpus, sh["lo"], sh["hi"]),
                                sh["hi"] + 1), parallelism=f"shard{args.gpus} (sequences per rank)")
    sample = smp.describe()
    line = {"metric": "decode tokens/s", "value": round(value, 3), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
            "impl": "reference", "config": config,
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample + "; C restatement of the reference's Java CPU attention "
                                                "(no JDK on this machine)"},
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ main arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="c5", choices=sorted(WORKLOADS))
    ap.add_argument("--no-suite", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="override the batch (profiling captures only)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist
    import b200attn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    if not os.path.exists(b200attn.LIB_PATH):
        if rank == 0:
            b200attn.build()
        if world > 1:
            dist.barrier()
    ctx = b200attn.Context(local)
    # decode layers start while the kernel ahead of them finishes (b2a_set_decode_early_start):
    # nothing launched here writes ctx_lens or the cache rows a decode reads right before it
    ctx.set_decode_early_start(True)
    hbm, tflops, src = peaks()

    if args.workload == "c3blk":
        if world > 1:
            raise SystemExit("--workload c3blk runs on one GPU")
        w = BlockWorkload()
    else:
        w = DecodeWorkload(args.workload, 5, args.batch, world, rank) if args.workload in ("c3", "c5") else \
            PrefillWorkload(args.workload, {"c1": 1, "c2": 2, "c4": 4}[args.workload], args.batch)
    for _ in range(args.warmup):
        w.step(ctx)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timed region: CUDA graph replays of the same launches
    # (one graph per decode layer, one per prefill step), captured after warm-up
    if isinstance(w, DecodeWorkload):
        graphs = [capture_graph(torch, (lambda i=i: w.launch(ctx, i))) for i in range(len(w.layers))]
        run_layer = [(g.replay if g is not None else (lambda i=i: w.launch(ctx, i))) for i, g in enumerate(graphs)]
    else:
        graphs = [capture_graph(torch, lambda: w.step(ctx))]
        run_step = graphs[0].replay if graphs[0] is not None else (lambda: w.step(ctx))
    launch_mode = "CUDA graph replay" if all(g is not None for g in graphs) else "direct launches"
    s = torch.cuda.current_stream()
    per_launch = []
    barrier()
    with NvmlClockSampler(local) as clk, ClockSampler(local) as clk_smi:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(s)
        if isinstance(w, DecodeWorkload):
            evs = []
            for _ in range(args.steps):
                for i in range(len(w.layers)):
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record(s)
                    run_layer[i]()
                    b.record(s)
                    evs.append((a, b))
        else:
            evs = []
            for _ in range(args.steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(s)
                run_step()
                b.record(s)
                evs.append((a, b))
        t1.record(s)
        barrier()
    elapsed_ms = t0.elapsed_time(t1)
    per_launch = [a.elapsed_time(b) for a, b in evs]
    clocks = clk.summary() or clk_smi.summary()
    del graphs

    # ---- end-to-end timed region (host buffers, copies inside)
    if isinstance(w, DecodeWorkload):
        for _ in range(2):
            w.step_e2e(ctx)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            w.step_e2e(ctx)
        e1.record(s)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        h2d, d2h = w.e2e_bytes()
    else:
        e2e_ms, h2d, d2h = elapsed_ms, 0, 0

    # max over ranks (device-timed)
    from b200attn import sharding
    elapsed_ms, e2e_ms = sharding.max_over_ranks([elapsed_ms, e2e_ms])
    ms_step = elapsed_ms / args.steps
    tokens = w.tokens_per_step() * world
    value = tokens / (ms_step / 1e3)
    e2e_value = tokens / (e2e_ms / args.steps / 1e3)

    # roofline of the dominant kernel (decode: the split-KV kernel; bytes summed over launches)
    kern_ms = sum(per_launch)
    if isinstance(w, DecodeWorkload):
        achieved = w.algorithmic_bytes() * args.steps / (kern_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": src + " (hbm_gbs, burst copy)",
                "kernel": "decode_tc_kernel<256,half>" if args.workload == "c5" else "decode_tc_kernel<64,half>",
                "bytes_per_step": w.algorithmic_bytes(), "traffic": None,
                "per_layer_ms": [round(statistics.mean(per_launch[i::len(w.layers)]), 4)
                                 for i in range(len(w.layers))]}
    elif isinstance(w, BlockWorkload):
        achieved = w.algorithmic_bytes() * args.steps / (kern_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": src + " (hbm_gbs, burst copy)",
                "kernel": "decode_tc_kernel<64,half> + linear_tc_kernel<128>", "bytes_per_step": w.algorithmic_bytes(),
                "traffic": None}
    else:
        achieved = w.flops() * args.steps / (kern_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4), "peak_source": src + " (bf16_tflops, burst)",
                "flops_per_step": w.flops(), "traffic": None}
    # DRAM traffic: ncu's dram__bytes_read + write cannot be read inside a timed run, so the committed
    # capture's ratio of traffic to algorithmic bytes is applied to this run's algorithmic bytes
    traffic_file = os.path.join(REPO, "profiles", f"decode_tc_kernel_{args.workload}_traffic.txt")
    if isinstance(w, DecodeWorkload) and os.path.exists(traffic_file):
        try:
            ratio = float(json.load(open(traffic_file))["traffic_over_algorithmic"])
            roof["traffic"] = int(round(ratio * w.algorithmic_bytes()))
            roof["traffic_source"] = (f"scaled: {ratio} x this step's algorithmic bytes, the ratio of "
                                      f"profiles/{os.path.basename(traffic_file)} (ncu dram__bytes_read.sum + "
                                      "dram__bytes_write.sum)")
        except Exception:
            pass

    line = {"metric": "decode tokens/s" if isinstance(w, DecodeWorkload) else "attn tokens/s",
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16" if isinstance(w, (DecodeWorkload, BlockWorkload)) else str(w.dt).split(".")[-1],
            "data": "synthetic (seeded N(0,1); no dataset or checkpoint)",
            "config": dict(w.config() if isinstance(w, DecodeWorkload) else {"workload": WORKLOADS[args.workload]},
                           parallelism=f"shard{world} (sequences per rank)", launch=launch_mode,
                           decode_early_start=True),
            "roofline": roof,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": w.kernel_launches_per_step() * args.steps,
            "clocks": clocks}

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, threads, secs, steps, sample = cpu_decode_sample(CPU_SAMPLE_SEQS, max_seconds=12.0)
        line["cpu_baseline"] = {"value": round(tps, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": f"{sample}, {steps} step(s) in {secs:.1f} s; C restatement of the "
                                          "reference's Java CPU attention (no JDK here)"}
    if rank == 0 and world == 1 and not args.no_suite:
        line["suite"] = run_suite(ctx, hbm, tflops, src)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
