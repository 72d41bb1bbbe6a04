"""DSA forward benchmark: query-tokens/s on 1..8 B200s, with per-stage rooflines.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

A step is one DSA forward (indexer -> top-K -> sparse attention) over one
batch of the workload, run through the C ABI of libdsa_b200.so.  Default
workload: config c5 (DeepSeek-V3.2 scale, B=1 T=32768 HI=64 DI=128 HQ=16
D=128 k=2048, bf16), the largest configuration that fits one GPU.

Scaling: "weak" (default) gives every rank its own sequences (batch
sharding); "strong" splits one workload's query rows across ranks (zig-zag
row blocks).  Neither communicates on the hot path.  Timing: W untimed
steps, then K steps between barrier + synchronize, CUDA events on the
launching stream, max over ranks.  Inputs are larger than L2 (c5: 0.9 GB of
inputs and a 4.3 GB score matrix per step), so no L2 flush is needed.

Rank 0 prints one JSON line.  ``--impl reference`` times the reference's
own CPU path (torch variant + the reference's AVX-512 top-K built in
oracle/_ref) on a bounded sample of the same workload's rows.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "dsa-cpu-topk_b200"))

CONFIGS = {
    # name: B, T, HI, DI, HQ, DQ(=DV), top_k, dtype, description
    "c1": dict(B=16, T=512, HI=4, DI=32, HQ=4, D=32, k=32, dtype="f32",
               desc="DSA fwd B16 T512 k32 HI4 DI32 HQ4 D32 fp32, causal"),
    "c3_b64_k128": dict(B=64, T=512, HI=4, DI=32, HQ=4, D=32, k=128, dtype="f32",
                        desc="DSA fwd B64 T512 k128 HI4 DI32 HQ4 D32 fp32, causal (c3 sweep corner)"),
    "c4": dict(B=4, T=8192, HI=16, DI=64, HQ=16, D=64, k=512, dtype="bf16",
               desc="DSA fwd B4 T8192 k512 HI16 DI64 HQ16 D64 bf16, causal"),
    "c5": dict(B=1, T=32768, HI=64, DI=128, HQ=16, D=128, k=2048, dtype="bf16",
               desc="DSA fwd B1 T32768 k2048 HI64 DI128 HQ16 D128 bf16, causal (DeepSeek-V3.2 scale)"),
    # c5 with the indexer inputs in FP8 (e4m3) as in the DeepSeek-V3.2 paper; not a BASELINE config
    "c5_fp8": dict(B=1, T=32768, HI=64, DI=128, HQ=16, D=128, k=2048, dtype="bf16", idx_dtype="fp8",
                   desc="c5 with e4m3 indexer q/k (FP8 indexer), bf16 Q/K/V"),
    # c5 with structured selections: indexer q/k carry a positional code, so each
    # query keeps a local window of keys plus strided "sink" blocks (most key
    # blocks of a query tile hold no kept key); not a BASELINE config
    "c5_local": dict(B=1, T=32768, HI=64, DI=128, HQ=16, D=128, k=2048, dtype="bf16", structured=True,
                     desc="c5 shapes, structured selections (local window + strided sink blocks), bf16"),
    # c5's head shapes at T=8192 (~2 GB on the device): the small case the ncu captures use
    "c5_t8k": dict(B=1, T=8192, HI=64, DI=128, HQ=16, D=128, k=2048, dtype="bf16",
                   desc="c5 head shapes at T8192 (profiling case), bf16, causal"),
    # rows longer than 8K, as at c5 (the top-K kernel's uncached variant), ~2.5 GB on the device
    "c5_t16k": dict(B=1, T=16384, HI=64, DI=128, HQ=16, D=128, k=2048, dtype="bf16",
                    desc="c5 head shapes at T16384 (profiling case), bf16, causal"),
}
DT = {"f32": torch.float32, "bf16": torch.bfloat16, "fp8": torch.float8_e4m3fn}
C2 = dict(B=64, T=2048, k=128, desc="top-K only: fp32 scores 64 x 2048 x 2048, N(0,1), s > t = -inf, k=128")


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes from committed ncu summaries (profiles/traffic.json)."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.gpu = vis.split(",")[local_rank] if vis else str(local_rank)
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        # Samples every 50 ms; the median is taken over the samples drawn under
        # load (board power at least half of the run's highest sample), so the
        # idle moments before and after the timed region do not count.
        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 9:
                    continue
                try:
                    sm_v, mx_v = float(c[1].split()[0]), float(c[2].split()[0])
                except ValueError:
                    continue
                try:
                    pw = float(c[3].split()[0])
                except ValueError:
                    pw = None
                rows.append((sm_v, mx_v, pw, [n for n, v in zip(names, c[5:9]) if v.lower().startswith("active")]))
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": []}
        pmax = max((r[2] for r in rows if r[2] is not None), default=None)
        load = [r for r in rows if pmax is None or (r[2] is not None and r[2] >= 0.5 * pmax)] or rows
        reasons = sorted({n for r in load for n in r[3]})
        return {"sm_mhz": statistics.median(r[0] for r in load),
                "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(load), "samples_all": len(rows),
                "power_w_median": statistics.median(r[2] for r in load) if pmax is not None else None,
                "reasons": reasons}


# --------------------------------------------------------------------------
# workload
# --------------------------------------------------------------------------

def make_inputs_device(cfg, B, dev, seed):
    """Seeded synthetic inputs of the config's shapes (N(0,1); w ~ N(0,1)/sqrt(HI))."""
    g = torch.Generator(device=dev).manual_seed(seed)
    dt = DT[cfg["dtype"]]
    T, HI, DI, HQ, D = cfg["T"], cfg["HI"], cfg["DI"], cfg["HQ"], cfg["D"]

    def rnd(shape, scale=1.0, dtype=dt):
        return (torch.randn(shape, generator=g, device=dev) * scale).to(dtype)

    it = DT[cfg.get("idx_dtype", cfg["dtype"])]
    if cfg.get("structured"):
        # positional code: <q_t, k_s> = mean_i cos(2 pi (t - s) / lambda_i) peaks at s = t
        # and decays with distance; one more dimension lifts keys s % 4096 < 128
        nf = (DI - 2) // 2
        pos = torch.arange(T, device=dev, dtype=torch.float32)
        lam = 2.0 ** torch.linspace(6.0, math.log2(T), nf, device=dev)
        ang = 2 * math.pi * pos[:, None] / lam[None, :]
        enc = torch.cat([ang.cos(), ang.sin()], dim=1) / math.sqrt(nf)            # [T, 2 nf]
        sink = ((pos % 4096) < 128).float()[:, None] * 0.8
        kk = torch.cat([enc, sink, torch.zeros(T, 1, device=dev)], dim=1)
        qq = torch.cat([enc, torch.ones(T, 1, device=dev), torch.zeros(T, 1, device=dev)], dim=1)
        k_idx = (kk[None] + 0.02 * torch.randn((B, T, DI), generator=g, device=dev)).to(it)
        q_idx = (qq[None, :, None, :] + 0.02 * torch.randn((B, T, HI, DI), generator=g, device=dev)).to(it)
        w_idx = torch.rand((B, T, HI), generator=g, device=dev) / HI
        return (q_idx, k_idx, w_idx, rnd((B, T, HQ, D)), rnd((B, T, HQ, D)), rnd((B, T, HQ, D)))
    return (rnd((B, T, HI, DI), dtype=it), rnd((B, T, DI), dtype=it), rnd((B, T, HI), 1 / math.sqrt(HI), torch.float32),
            rnd((B, T, HQ, D)), rnd((B, T, HQ, D)), rnd((B, T, HQ, D)))


class Pipeline:
    """Preallocated buffers and the three C-ABI stage calls for some row blocks.

    Two equal row blocks of one sequence (a rank's zig-zag pair under strong
    scaling) run as ONE launch per stage: the blocks are stacked as a batch of
    2 with the key side shared (batch stride 0) and row_bstep = the distance
    between their first rows.  Anything else runs one launch per block."""

    def __init__(self, inputs, blocks, k):
        import _native
        from topk import idx_cap_for
        self.n = _native
        q, kk, w, Q, K, V = inputs
        B, T = Q.shape[:2]
        self.k = min(k, T)
        self.cap = idx_cap_for(self.k, T)
        self.parts = []
        dev = Q.device
        lens = {b.stop - b.start for b in blocks}
        self.stacked = len(blocks) == 2 and B == 1 and len(lens) == 1
        if self.stacked:
            a, b = blocks
            st = lambda x: torch.cat([x[:, a.start:a.stop], x[:, b.start:b.stop]]).contiguous()
            groups = [dict(q0=a.start, bstep=b.start - a.start, Tq=a.stop - a.start, NB=2,
                           q=st(q), w=st(w), Q=st(Q))]
            exp = lambda x: x.expand(2, *x.shape[1:])
            self.k_idx, self.K, self.V = exp(kk), exp(K), exp(V)
        else:
            groups = [dict(q0=blk.start, bstep=0, Tq=blk.stop - blk.start, NB=B,
                           q=q[:, blk.start:blk.stop].contiguous(), w=w[:, blk.start:blk.stop].contiguous(),
                           Q=Q[:, blk.start:blk.stop].contiguous()) for blk in blocks]
            self.k_idx, self.K, self.V = kk, K, V
        for p in groups:
            NB, Tq = p["NB"], p["Tq"]
            p.update(scores=torch.empty((NB, Tq, T), device=dev, dtype=torch.float32),
                     thr=torch.empty(NB * Tq, device=dev, dtype=torch.float32),
                     cnt=torch.empty(NB * Tq, device=dev, dtype=torch.int32),
                     idx=torch.empty((NB * Tq, self.cap), device=dev, dtype=torch.int32),
                     O=torch.empty((NB, Tq, Q.shape[2], V.shape[3]), device=dev, dtype=torch.float32))
            self.parts.append(p)
        # stage 3 on the tensor cores (kept-set bitmap + masked flash attention)
        # where the dtype and head size allow, else the gather over kept lists
        self.tc = _native.attn_tc_supported(Q, V) and os.environ.get("DSA_ATTN_GATHER") != "1"
        self.words = _native.bitmap_words(T)
        self.v16 = False
        if self.tc:
            for p in self.parts:
                p["bits"] = torch.empty((p["NB"] * p["Tq"], self.words), device=dev, dtype=torch.int32)
                # the top-K's candidate lists (sweep + resolve kernels)
                p["tws"] = torch.empty(_native.topk_select_bitmap_workspace_bytes(p["NB"] * p["Tq"], self.words),
                                       device=dev, dtype=torch.uint8)
                # stage 3's workspace: block summary, fp16 copy of V (bf16)
                nws = _native.sparse_attn_bitmap_workspace_bytes(p["NB"], p["Tq"], T, Q.shape[2], V.shape[3],
                                                                 _native.dtype_code(Q))
                p["ws"] = torch.empty(nws, device=dev, dtype=torch.uint8) if nws else None
                self.v16 = self.v16 or bool(nws)
        self.stage_names = ["indexer", "topk", "sparse_attn"]
        # stage 3 with its workspace: block summary (+ |V| max and fp16 conversion
        # for bf16) + attention
        v16 = self.tc and Q.dtype == torch.bfloat16
        # the bitmap top-K of rows longer than 4K (up to 32K) is two kernels (sweep + resolve)
        two = sum(1 for p in self.parts
                  if 4096 < min(T, p["q0"] + (p["NB"] - 1) * p["bstep"] + p["Tq"]) <= 32768) if self.tc else 0
        self.launches_per_step = (len(self.stage_names) + (1 if self.v16 else 0) + (2 if v16 else 0)) * \
            len(self.parts) + two
        # opt-in one-launch kernel for short sequences (DSA_FUSED_SMALL=1)
        self.fused = T <= 2048 and bool(os.environ.get("DSA_FUSED_SMALL")) and not self.stacked
        if self.fused:
            from dsa_attention import forward_workspace_bytes
            self.ws = [torch.empty(forward_workspace_bytes(B, p["Tq"], T, self.k), device=dev, dtype=torch.uint8)
                       for p in self.parts]
            self.launches_per_step = len(self.parts)
            self.stage_names = ["fused_forward"]
        self.step(None)  # untimed: fills the kept counts used for accounting
        for p in self.parts:
            NB, Tq, T = p["scores"].shape
            if self.tc or self.fused:
                self.n.topk_select_ex(p["scores"], NB * Tq, T, T, self.k, p["thr"], None, p["cnt"], 0,
                                      causal=True, rows_per_batch=Tq, q_row0=p["q0"], row_bstep=p["bstep"])

    def out_rows(self):
        """This rank's output rows in block order, [B, rows, HQ, D]."""
        if self.stacked:
            O = self.parts[0]["O"]
            return torch.cat([O[0:1], O[1:2]], dim=1)
        return torch.cat([p["O"] for p in self.parts], dim=1)

    def step(self, ev=None):
        """One forward over every row block; ev[i][j] brackets stage j of part i."""
        n = self.n
        for i, p in enumerate(self.parts):
            rec = (lambda j: ev[i][j].record()) if ev is not None else (lambda j: None)
            rec(0)
            if self.fused:
                n.forward(p["q"], self.k_idx, p["w"], p["Q"], self.K, self.V, p["O"], self.k, self.ws[i],
                          q_row0=p["q0"])
                rec(1)
                continue
            q0, bs = p["q0"], p["bstep"]
            n.indexer_scores_ex(p["q"], self.k_idx, p["w"], p["scores"], q_row0=q0, row_bstep=bs,
                                fill_upper=False)
            rec(1)
            NB, Tq, T = p["scores"].shape
            if self.tc:
                n.topk_select_bitmap(p["scores"], self.k, p["thr"], p["bits"], causal=True, q_row0=q0,
                                     row_bstep=bs, workspace=p["tws"])
                rec(2)
                n.sparse_attn_bitmap_ex(p["bits"], p["Q"], self.K, self.V, p["O"], q_row0=q0, row_bstep=bs,
                                        workspace=p["ws"])
                rec(3)
                continue
            n.topk_select_ex(p["scores"], NB * Tq, T, T, self.k, p["thr"], p["idx"], p["cnt"], self.cap,
                             causal=True, rows_per_batch=Tq, q_row0=q0, row_bstep=bs)
            rec(2)
            n.sparse_attn_ex(p["idx"], p["cnt"], self.cap, p["scores"], p["thr"], p["Q"], self.K, self.V,
                             p["O"], q_row0=q0, row_bstep=bs)
            rec(3)

    def algorithmic(self, cfg):
        """Per-step algorithmic work of each stage (from the actual kept counts)."""
        elt = 2 if cfg["dtype"] == "bf16" else 4
        HI, DI, HQ, D = cfg["HI"], cfg["DI"], cfg["HQ"], cfg["D"]
        flops = topk_b = attn_b = attn_f = tile_f = 0
        for p in self.parts:
            NB, Tq, T = p["scores"].shape
            rows = NB * Tq
            sel = p["cnt"].double().sum().item()
            for bb in range(NB):
                r0 = p["q0"] + bb * p["bstep"]          # this batch's first query row
                t = torch.arange(r0, r0 + Tq, dtype=torch.float64)
                valid = torch.clamp(t + 1, max=T).sum().item()
                flops += 2.0 * HI * DI * valid
                topk_b += 4.0 * valid
                # tensor-core stage 3: every 128x128 (query, key) tile up to the
                # diagonal is two MMAs of 2*128*128*D FLOPs per head; with its
                # workspace the kernel skips the key blocks that hold no kept key
                # of the query tile, so those are counted from the bitmap
                if self.tc and p.get("ws") is not None:
                    nbk = self.words // 4
                    kb = p["bits"][bb * Tq:(bb + 1) * Tq].view(Tq, nbk, 4).ne(0).any(-1)
                    pad = (-Tq) % 128
                    if pad:
                        kb = torch.cat([kb, kb.new_zeros((pad, nbk))])
                    tile_f += HQ * 4.0 * 128 * 128 * D * kb.view(-1, 128, nbk).any(1).sum().item()
                    continue
                for qt in range((Tq + 127) // 128):
                    t_end = r0 + min((qt + 1) * 128, Tq)
                    nblk = min((t_end - 1) // 128 + 1, (T + 127) // 128)
                    tile_f += HQ * nblk * 4.0 * 128 * 128 * D
            topk_b += (4.0 * rows + 4.0 * rows * self.words if self.tc else 8.0 * rows + 4.0 * sel)
            attn_b += sel * HQ * 2 * D * elt + rows * HQ * D * (elt + 4) + 4.0 * sel + 4.0 * rows
            attn_f += sel * HQ * 4.0 * D
        return dict(indexer_flops=flops, topk_bytes=topk_b, attn_bytes=attn_b, attn_flops=attn_f,
                    attn_tile_flops=tile_f)


# --------------------------------------------------------------------------
# the reference's CPU path (timed baseline; oracle/ is used only here)
# --------------------------------------------------------------------------

def cpu_reference_setup(cfg, inputs):
    """Host copies of one sequence (batch 0) and the reference's compiled top-K."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import build_ref
    import dsa_oracle
    ext = build_ref.load_ref()
    host = [x[:1].float().cpu() for x in inputs]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return dict(ext=ext, oracle=dsa_oracle, host=host, threads=threads)


def cpu_reference_rows(ctx, cfg, rows: range):
    """The reference torch variant's work for query rows ``rows`` of one sequence:
    dense indexer einsum over all T keys (lightning_indexer.py:26-33), k-th
    largest per row (the reference's AVX-512 topk_threshold, else torch.topk)
    and the dense masked softmax attention (dsa_attention.py:46-51)."""
    o = ctx["oracle"]
    q, kk, w, Q, K, V = ctx["host"]
    a, z = rows.start, rows.stop
    s = o.indexer_scores(q, kk, w, slice(a, z))
    k_eff = min(cfg["k"], s.shape[-1])
    thr = ctx["ext"].topk_threshold(s.contiguous(), k_eff) if ctx["ext"] is not None \
        else o.select_threshold(s, k_eff)
    return o._attend(s, thr, Q, K, V, a, z, 1.0 / math.sqrt(cfg["D"]))


def cpu_reference_rate(ctx, cfg, seconds: float, chunk: int):
    """Query rows/s of the reference CPU path over a bounded sample of rows
    spread across the sequence (the torch variant's cost per row does not
    depend on t: it scores every key and masks)."""
    T = cfg["T"]
    starts = list(range(0, T - chunk + 1, max(chunk, (T // 64) // chunk * chunk or chunk)))
    cpu_reference_rows(ctx, cfg, range(starts[0], starts[0] + chunk))    # warm-up
    done, t0 = 0, time.perf_counter()
    i = 0
    while True:
        a = starts[(i * 37) % len(starts)]
        cpu_reference_rows(ctx, cfg, range(a, a + chunk))
        done += chunk
        i += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= T * cfg["B"]:
            return done / el, done, el


def cpu_kind(ctx):
    """"port": the indexer and attention legs are this repo's restatement of the
    reference's torch variant; only the top-K leg is the reference's own code."""
    return "port"


def cpu_extra(ctx, cfg, rows):
    """What the CPU number is made of, and that it is a rate over sampled rows."""
    return {"components": {
                "indexer": "port: oracle/dsa_oracle.py restatement of lightning_indexer.py:26-33 (torch, fp32)",
                "topk": ("reference: topk_avx512.cpp compiled from its sources (oracle/_ref)"
                         if ctx["ext"] is not None else "port: torch.topk (AVX-512 extension unavailable)"),
                "attention": "port: oracle/dsa_oracle.py restatement of dsa_attention.py:46-51 (torch, fp32)"},
            "extrapolated": True, "rows_sampled": int(rows), "rows_per_step": cfg["B"] * cfg["T"]}


def cpu_sample_text(ctx, cfg, rows, el):
    topk = ("the reference's topk_avx512.cpp built from its sources in oracle/_ref"
            if ctx["ext"] is not None else "torch.topk (AVX-512 extension unavailable on this host)")
    return (f"{rows} query rows of {cfg['desc']} in {el:.1f} s; dense indexer + masked softmax as "
            f"the reference torch variant (restated in oracle/dsa_oracle.py, fp32 upcast), top-K by {topk}; "
            f"OMP/torch threads={ctx['threads']}")


CHUNK = {"c1": 512, "c3_b64_k128": 512, "c4": 64, "c5": 16, "c5_local": 16, "c5_fp8": 16, "c5_t8k": 32,
         "c5_t16k": 32}


# --------------------------------------------------------------------------
# arms
# --------------------------------------------------------------------------

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def base_line(args, cfg, world, value, ms, unit="query-tokens/s"):
    B_glob = cfg["B"] * (world if args.scaling == "weak" else 1)
    return {
        "metric": "DSA fwd query-tokens/s",
        "value": value, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded N(0,1) inputs of the config's shapes)",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "global_batch": B_glob,
                   "seq_len": cfg["T"], "top_k": cfg["k"], "HI": cfg["HI"], "DI": cfg["DI"],
                   "HQ": cfg["HQ"], "D": cfg["D"],
                   "parallelism": (f"batch-shard x{world}" if args.scaling == "weak"
                                   else f"query-row zig-zag x{world}"),
                   "row_blocks": ("each rank: its own whole sequences" if args.scaling == "weak" else
                                  "one sequence; rank r owns row blocks r and 2N-1-r of 2N, run as one "
                                  "launch per stage (B=2 row blocks, shared key side)" if world > 1 else
                                  "one sequence, all rows on one GPU"),
                   "l2": "inputs larger than L2" if cfg["T"] >= 8192 else
                         "L2 flushed between steps (256 MB write)"},
    }


def run_b200(args, cfg, world, rank, local):
    import sharding
    from dsa_attention import dsa_forward, forward_workspace_bytes
    dev = torch.device("cuda", local)
    B, T = cfg["B"], cfg["T"]
    seed = 1000 * (rank if args.scaling == "weak" else 0)
    inputs = make_inputs_device(cfg, B, dev, seed)
    if args.scaling == "weak" or world == 1:
        blocks = [sharding.RowBlock(0, T)]
    else:
        blocks = sharding.zigzag_plan(T, world)[rank]
    pipe = Pipeline(inputs, blocks, cfg["k"])
    flush = None if T >= 8192 else torch.empty(256 << 20, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        pipe.step()
    nb = len(pipe.parts)
    ns = len(pipe.stage_names)
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(ns + 1)] for _ in range(nb)]
           for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total_ms = 0.0
    if flush is None:
        start.record(stream)
        for s in range(args.steps):
            pipe.step(evs[s])
        end.record(stream)
        barrier(world)
        total_ms = start.elapsed_time(end)
    else:
        # small workloads: flush L2 between steps, time only the steps.  The
        # step is replayed from a CUDA graph, so host launch latency (three
        # ctypes calls) does not idle the GPU inside the timed region; the
        # per-stage split then comes from eager steps after the timing.
        graph = None
        if not os.environ.get("DSA_BENCH_NO_GRAPH"):
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    pipe.step()
                graph.replay()
                torch.cuda.synchronize()
            except Exception as e:  # capture is an optimisation of the timing only
                print(f"bench: CUDA graph capture failed ({e}); timing eager steps", file=sys.stderr)
                graph = None
        for s in range(args.steps):
            flush.zero_()
            start.record(stream)
            if graph is not None:
                graph.replay()
            else:
                pipe.step(evs[s])
            end.record(stream)
            end.synchronize()
            total_ms += start.elapsed_time(end)
        barrier(world)
        if graph is not None:
            for s in range(args.steps):
                flush.zero_()
                pipe.step(evs[s])
            torch.cuda.synchronize()
        pipe.graph = graph is not None
    clk = clocks.stop()
    stage_ms = [0.0] * ns
    for s in range(args.steps):
        for i in range(nb):
            for j in range(ns):
                stage_ms[j] += evs[s][i][j].elapsed_time(evs[s][i][j + 1])
    stage_ms = [x / args.steps for x in stage_ms]
    t_max = max_over_ranks(total_ms, world)
    ms = t_max / args.steps
    tokens = B * T * (world if args.scaling == "weak" else 1)
    value = tokens / (ms / 1e3)

    # rooflines of each stage (algorithmic work / measured average duration)
    hbm, tflops, src = load_peaks()
    peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if src == "measured" else {}
    tf_sust = peaks.get("bf16_tflops_sustained", 1400.0 if src == "fallback" else tflops)
    # The bf16 denominator follows the clocks this run saw: the burst GEMM peak
    # when the SM clock stayed within 5% of its maximum (a burst), else the
    # sustained (power-capped) one.  Both fractions are reported.
    at_max = bool(clk.get("sm_mhz") and clk.get("sm_max_mhz") and clk["sm_mhz"] >= 0.95 * clk["sm_max_mhz"])
    tf_peak = tflops if at_max else tf_sust
    tf_label = (f"burst bf16 GEMM peak ({'measured' if src == 'measured' else 'fallback'}; SM clock median "
                f"{clk.get('sm_mhz')} of {clk.get('sm_max_mhz')} MHz)" if at_max else
                "sustained bf16 GEMM peak (SM clock below 95% of max)")
    alg = pipe.algorithmic(cfg)
    traffic = load_traffic().get(args.config, {})
    if pipe.fused:
        stages = {}   # filled below
    else:
        stages = {
            "indexer": dict(bound="tensor", achieved=alg["indexer_flops"] / (stage_ms[0] / 1e3) / 1e12,
                            peak=tf_peak * (2 if cfg.get("idx_dtype") == "fp8" else 1), unit="TFLOP/s",
                            ms=stage_ms[0],
                            kernel=("indexer_tc (e4m3, kind::f8f6f4)" if cfg.get("idx_dtype") == "fp8" else
                                    "indexer_tc" if cfg["dtype"] == "bf16" else "indexer_simt (fp32 CUDA cores)"),
                            traffic=traffic.get("indexer")),
            "topk": dict(bound="hbm", achieved=alg["topk_bytes"] / (stage_ms[1] / 1e3) / 1e9, peak=hbm,
                         unit="GB/s", ms=stage_ms[1], kernel="topk_select_kernel", traffic=traffic.get("topk")),
            "sparse_attn": dict(bound="hbm", achieved=alg["attn_bytes"] / (stage_ms[-1] / 1e3) / 1e9, peak=hbm,
                                unit="GB/s", ms=stage_ms[-1], kernel="sparse_attn_kernel",
                                traffic=traffic.get("sparse_attn")),
        }
        if pipe.tc:
            stages["topk"]["kernel"] = "topk_sweep_kernel + topk_resolve_kernel (threshold + kept-set bitmap)"
            stages["sparse_attn"] = dict(
                bound="tensor", achieved=alg["attn_tile_flops"] / (stage_ms[2] / 1e3) / 1e12, peak=tf_peak,
                unit="TFLOP/s", ms=stage_ms[2], kernel="attn_tc2_kernel", traffic=traffic.get("sparse_attn"),
                note="FLOPs of the 128x128 (query, key) tiles (QK^T and PV) the masked flash attention runs: the causal tiles holding a kept key",
                useful_tflops=alg["attn_flops"] / (stage_ms[2] / 1e3) / 1e12,
                useful_fraction_of_tile_flops=alg["attn_flops"] / max(alg["attn_tile_flops"], 1.0))
            stages["sparse_attn"]["useful_frac"] = stages["sparse_attn"]["useful_tflops"] / tf_peak
        for v in stages.values():
            v["frac"] = v["achieved"] / v["peak"]
            if v["unit"] == "TFLOP/s":
                mult = 2 if v is stages.get("indexer") and cfg.get("idx_dtype") == "fp8" else 1
                v["frac_of_burst"] = v["achieved"] / (tflops * mult)
                v["frac_of_sustained"] = v["achieved"] / (tf_sust * mult)
                v["peak_source"] = tf_label + (" (MEASURED_PEAKS.json)" if src == "measured" else "")
            else:
                v["peak_source"] = "measured copy bandwidth (MEASURED_PEAKS.json)" if src == "measured" else "fallback"
    if cfg.get("idx_dtype") == "fp8" and not pipe.fused:
        stages["indexer"]["peak_source"] += "; FP8 peak taken as 2x the bf16 one (none measured)"
    if pipe.fused:
        elt = 2 if cfg["dtype"] == "bf16" else 4
        io = sum(x.numel() * x.element_size() for x in inputs[:4]) + B * T * cfg["HQ"] * cfg["D"] * 4
        fb = io + alg["attn_bytes"]
        stages = {"fused_forward": dict(bound="hbm", achieved=fb / (stage_ms[0] / 1e3) / 1e9, peak=hbm,
                                        unit="GB/s", ms=stage_ms[0], kernel="fused_small_kernel",
                                        traffic=traffic.get("fused_forward"),
                                        frac=fb / (stage_ms[0] / 1e3) / 1e9 / hbm,
                                        peak_source=f"{src} (MEASURED_PEAKS.json)",
                                        note="one launch: indexer + top-K + attention; bytes = inputs + O + "
                                             "gathered K/V rows (mostly L2-served)")}
    top = max(stages, key=lambda n: stages[n]["ms"])
    roof = {k2: stages[top][k2] for k2 in ("bound", "achieved", "peak", "unit", "frac", "traffic")}
    roof["kernel"] = top

    line = base_line(args, cfg, world, value, ms)
    line["roofline"] = roof
    line["stages"] = stages
    line["algorithmic"] = alg
    line["clocks"] = clk
    line["gpu_launches"] = pipe.launches_per_step * args.steps
    if getattr(pipe, "graph", False):
        line["timing"] = ("each timed step replays a CUDA graph of the stage launches; the stage split "
                          "comes from eager steps after the timed region")

    # ---- end to end through the public API: pinned host inputs -> device -> O back to host.
    # Every step copies its inputs in from pinned host memory and its output back
    # out.  As in a serving loop, steps are pipelined over two device buffer sets:
    # step i+1's host->device copies (copy-in stream) and step i-1's
    # device->host copy (copy-out stream) overlap step i's kernels.
    # Each rank copies only its own query rows.  With several ranks sharing one
    # sequence, the key side (k_idx, K, V) crosses PCIe once: every rank copies
    # 1/N of its rows and one NCCL all_gather over NVLink assembles the rest.
    if not args.no_e2e:
        q, kk, w, Q, K, V = inputs
        share_keys = args.scaling == "strong" and world > 1 and T % world == 0
        key_full = [x for x in (kk, K, V)]
        if share_keys:
            rows_r = slice(rank * (T // world), (rank + 1) * (T // world))
            h_key = [x[:, rows_r].cpu().pin_memory() for x in key_full]
        else:
            h_key = [x.cpu().pin_memory() for x in key_full]
        h_rows = [[p[name].cpu().pin_memory() for name in ("q", "w", "Q")] for p in pipe.parts]
        NSLOT = 2
        d_key = [[torch.empty_like(x, device=dev) for x in key_full] for _ in range(NSLOT)]
        d_chunk = [[torch.empty_like(x, device=dev) for x in h_key] for _ in range(NSLOT)] if share_keys else None
        d_rows = [[[torch.empty_like(x, device=dev) for x in r] for r in h_rows] for _ in range(NSLOT)]
        ws = [[torch.empty(max(1, forward_workspace_bytes(p["NB"], p["Tq"], T, cfg["k"], cfg["HQ"], cfg["D"],
                                                          Q.dtype)), device=dev, dtype=torch.uint8)
               for p in pipe.parts] for _ in range(NSLOT)]
        h_out = [[torch.empty(tuple(p["O"].shape), dtype=torch.float32).pin_memory() for p in pipe.parts]
                 for _ in range(NSLOT)]
        bi = sum(x.numel() * x.element_size() for x in h_key) + \
            sum(x.numel() * x.element_size() for r in h_rows for x in r)
        bo = sum(x.numel() * x.element_size() for x in h_out[0])
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev = lambda: torch.cuda.Event()
        comp_done = [ev() for _ in range(NSLOT)]
        in_done = [ev() for _ in range(NSLOT)]
        used = [False] * NSLOT
        if share_keys:
            import torch.distributed as dist

        def e2e_step(i):
            sl = i % NSLOT
            with torch.cuda.stream(s_in):
                if used[sl]:
                    s_in.wait_event(comp_done[sl])   # the slot's previous step has read its inputs
                if share_keys:
                    for c, h, full in zip(d_chunk[sl], h_key, d_key[sl]):
                        c.copy_(h, non_blocking=True)
                        # [1, T, ...] from N chunks of [1, T/N, ...] (dimension 0 of the flat views)
                        dist.all_gather_into_tensor(full.view(T, -1), c.view(T // world, -1))
                else:
                    for d, h in zip(d_key[sl], h_key):
                        d.copy_(h, non_blocking=True)
                for dr, hr in zip(d_rows[sl], h_rows):
                    for d, h in zip(dr, hr):
                        d.copy_(h, non_blocking=True)
                in_done[sl].record(s_in)
            stream.wait_event(in_done[sl])
            outs = []
            for j, p in enumerate(pipe.parts):
                qd, wd, Qd = d_rows[sl][j]
                outs.append(dsa_forward(qd, d_key[sl][0], wd, Qd, d_key[sl][1], d_key[sl][2], cfg["k"],
                                        q_row0=p["q0"], row_bstep=p["bstep"], workspace=ws[sl][j]))
            comp_done[sl].record(stream)
            used[sl] = True
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[sl])
                for j, o in enumerate(outs):
                    o.record_stream(s_out)
                    h_out[sl][j].copy_(o, non_blocking=True)

        for i in range(max(1, args.warmup)):
            e2e_step(i)
        s_in.synchronize(); s_out.synchronize()
        barrier(world)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(s_in)
        stream.wait_event(e_start)
        for i in range(args.steps):
            e2e_step(i)
        s_out.wait_stream(stream)
        e_end.record(s_out)
        e_end.synchronize()
        barrier(world)
        e_ms = max_over_ranks(e_start.elapsed_time(e_end), world) / args.steps
        h2d = max_over_ranks(float(bi), world) if world > 1 else bi
        line["e2e"] = {"value": tokens / (e_ms / 1e3), "unit": "query-tokens/s", "ms_per_step": e_ms,
                       "h2d_bytes_per_step": sum_over_ranks(bi, world),
                       "d2h_bytes_per_step": sum_over_ranks(bo, world),
                       "h2d_bytes_per_step_max_rank": h2d,
                       "api": "dsa_attention.dsa_forward (C ABI dsa_forward_ex), pinned host buffers, "
                              "copies of neighbouring steps overlapped on two streams" +
                              ("; key side copied 1/N per rank and all-gathered over NVLink (NCCL) "
                               "before the forward" if share_keys else "")}
        line["gpu_launches"] += pipe.launches_per_step * args.steps
        del h_key, h_rows, d_key, d_rows, ws, h_out, d_chunk

    # ---- verification (outside every timed region): gather the sharded rows over
    # NCCL and compare them with rank 0's own single-GPU forward of the whole
    # workload.  Both run the same kernels, so the rows must match bit for bit.
    if args.scaling == "strong" and not args.no_verify:
        from dsa_attention import dsa_forward as fwd_all
        plan = [blocks] if world == 1 else sharding.zigzag_plan(T, world)
        local_rows = pipe.out_rows()
        full = sharding.gather_rows(local_rows, plan) if world > 1 else local_rows
        if rank == 0:
            whole = fwd_all(*inputs, cfg["k"])
            line["verify"] = {"rows": T, "max_abs_diff": float((full - whole).abs().max()),
                              "bitwise_equal": bool(torch.equal(full, whole)),
                              "gather": "NCCL all_gather of output rows" if world > 1 else "none (1 rank)"}
        del full

    # ---- CPU baseline (rank 0 at N=1 only)
    if world == 1 and rank == 0 and not args.no_cpu:
        ctx = cpu_reference_setup(cfg, inputs)
        rate, rows, el = cpu_reference_rate(ctx, cfg, args.cpu_seconds, CHUNK[args.config])
        line["cpu_baseline"] = {"value": rate, "unit": "query-tokens/s", "cores": ctx["threads"],
                                "kind": cpu_kind(ctx), "sample": cpu_sample_text(ctx, cfg, rows, el),
                                **cpu_extra(ctx, cfg, rows)}
    return line


def run_topk_only(args, world, rank, local):
    """Config c2: stage 2 alone, rows/s (one row = one query's 2048 scores)."""
    import _native
    from topk import idx_cap_for
    dev = torch.device("cuda", local)
    B, T, k = C2["B"], C2["T"], C2["k"]
    g = torch.Generator(device=dev).manual_seed(1000 * rank)
    s = torch.randn((B, T, T), generator=g, device=dev)
    s.masked_fill_(~torch.ones(T, T, device=dev, dtype=torch.bool).tril(), float("-inf"))
    rows = B * T
    cap = idx_cap_for(k, T)
    thr = torch.empty(rows, device=dev)
    cnt = torch.empty(rows, device=dev, dtype=torch.int32)
    idx = torch.empty((rows, cap), device=dev, dtype=torch.int32)
    flush = torch.empty(256 << 20, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream()
    res = {}
    for mode in ("full", "causal"):
        def step():
            _native.topk_select(s, rows, T, T, k, thr, idx, cnt, cap, causal=(mode == "causal"),
                                rows_per_batch=T)
        for _ in range(args.warmup):
            step()
        barrier(world)
        tot = 0.0
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(args.steps):
            flush.zero_()
            st.record(stream); step(); en.record(stream); en.synchronize()
            tot += st.elapsed_time(en)
        ms = max_over_ranks(tot, world) / args.steps
        read = rows * T * 4 if mode == "full" else B * T * (T + 1) / 2 * 4
        written = rows * 8 + cnt.double().sum().item() * 4
        res[mode] = dict(ms=ms, rows_per_s=world * rows / (ms / 1e3), gbs=(read + written) / (ms / 1e3) / 1e9)
    hbm, _, src = load_peaks()
    line = {"metric": "top-K rows/s (per-row k-th largest + kept-index list)", "value": res["full"]["rows_per_s"],
            "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["full"]["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": {"workload": f"c2: {C2['desc']}",
                                                             "l2": "L2 flushed between steps (256 MB write)"},
            "roofline": {"bound": "hbm", "achieved": res["full"]["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": res["full"]["gbs"] / hbm, "traffic": None, "kernel": "topk_select"},
            "causal_mode": res["causal"], "gpu_launches": 2 * (args.steps + args.warmup)}
    if world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import build_ref
        ext = build_ref.load_ref()
        sample = s[:4].cpu().contiguous()                      # 8192 rows
        f = (lambda x: ext.topk_threshold(x, k)) if ext else (lambda x: x.topk(k, -1).values[..., -1:])
        f(sample)
        t0 = time.perf_counter(); n = 0
        while time.perf_counter() - t0 < args.cpu_seconds:
            f(sample); n += 1
        el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": n * sample.shape[0] * T / el, "unit": "rows/s",
                                "cores": torch.get_num_threads(),
                                "kind": "reference" if ext else "port",
                                "sample": f"{n} x 8192 rows of 2048 (threshold only, as topk_threshold) in {el:.1f} s"}
    return line


def run_reference(args, cfg, world, rank, local):
    """The reference's own CPU implementation of the path on this host's cores."""
    dev = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    inputs = make_inputs_device(cfg, 1, dev, 0)
    ctx = cpu_reference_setup(cfg, inputs)
    del inputs
    chunk = CHUNK[args.config]
    r1, _, el1 = cpu_reference_rate(ctx, cfg, 0.0, chunk)          # probe one chunk
    per_row = 1.0 / r1
    step_rows = max(chunk, int(args.ref_step_seconds / per_row) // chunk * chunk)
    step_rows = min(step_rows, cfg["T"] - cfg["T"] % chunk or chunk)
    starts = list(range(0, cfg["T"] - step_rows + 1, chunk)) or [0]

    def step(i):
        a = starts[(i * 7919) % len(starts)]
        for c in range(a, a + step_rows, chunk):
            cpu_reference_rows(ctx, cfg, range(c, min(c + chunk, cfg["T"])))

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    el = time.perf_counter() - t0
    value = step_rows * args.steps / el
    line = base_line(args, cfg, world, value, el / args.steps * 1e3)
    line["impl"] = "reference"
    line["n_gpus"] = world
    line["cpu_baseline"] = {"value": value, "unit": "query-tokens/s", "cores": ctx["threads"],
                            "kind": cpu_kind(ctx),
                            "sample": cpu_sample_text(ctx, cfg, step_rows * args.steps, el) +
                            f"; {step_rows} rows per step",
                            **cpu_extra(ctx, cfg, step_rows * args.steps)}
    line["e2e"] = {"value": value, "unit": "query-tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    line["gpu_launches"] = 0
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS) + ["c2"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--scaling", default="auto", choices=["auto", "weak", "strong"],
                    help="auto: strong (one sequence's query rows split zig-zag over the ranks) when the "
                         "config has one sequence (c5) or fewer sequences than ranks, else weak")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-step-seconds", type=float, default=3.0)
    ap.add_argument("--no-verify", action="store_true",
                    help="skip the check after timing (strong scaling): gather the sharded output rows "
                         "(NCCL) and compare them with a single-GPU forward on rank 0")
    args = ap.parse_args()
    cfg = CONFIGS.get(args.config)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.scaling == "auto":
        args.scaling = "strong" if cfg is not None and (cfg["B"] == 1 or cfg["B"] < world) else "weak"
    if args.config == "c2":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "c2 is a top-K-only config; its CPU "
                              "baseline is reported in the b200 arm's cpu_baseline"}), flush=True)
            return
        world, rank, local = dist_setup()
        line = run_topk_only(args, world, rank, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        line = run_reference(args, cfg, world, rank, int(os.environ.get("LOCAL_RANK", "0")))
        print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup()
    line = run_b200(args, cfg, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
