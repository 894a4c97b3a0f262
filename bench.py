#!/usr/bin/env python3
"""Benchmark: batch-1 Q8_0 decode of a LLaMA-2-7B-shape model on B200, plus the Q8_0 GEMV shapes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|gemv|gemm]

Decode workload (N=1): LLaMA-2-7B shape (dim 4096, hidden 11008, 32 layers, 32 heads, 32 KV heads,
vocab 32000, seq_len 4096), random-init weights N(0, 0.02) generated on the GPU from a seed, rounded
to bf16 and quantised to Q8_0 by the library's load-time quantiser; fp32 KV cache.  One step = a
seeded 32-token prompt whose 31 forced positions are prefilled in one batch on the tensor cores
(dk_model_prefill, on every rank under tensor parallelism), then 256 greedy tokens.
`value` = generated tokens per second of the 256-token decode phase, timed with CUDA events on the
engine's stream, inputs resident in HBM; the weights (7.4 GB) are far larger than L2, so every token
streams them from HBM.  `e2e` = the same tokens per second through the C-ABI generate entry point
(dk_model_generate: host prompt in, host tokens out, copies included), wall clock, prompt prefill
included.  `prefill` = dk_model_prefill of a 2048-token prompt (positions/s, int8 TOPS of its
matmuls); `prefill_gemm` = the tensor-core matmul alone on one layer's shapes at 256 positions.

Reference arm (--impl reference): the reference's own CPU forward (its unmodified sources compiled
with its own flags, oracle/_ref) on the host cores, on a bounded sample of the same workload: the
7B-shape model with 1 and with 3 layers (Q8_0 cache files written from the same distribution),
per-token time extrapolated linearly to 32 layers.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 32
GEN_LEN = 256


def _models():
    from diolkos_b200 import synth

    # name -> (shape, prompt positions, greedy tokens timed, label)
    return {"7b": (synth.LLAMA7B, PROMPT_LEN, GEN_LEN, "llama2-7b-shape"),
            "70b": (synth.LLAMA70B, 512, 128, "llama2-70b-shape")}
SEED = 20260
GEMV_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]  # [out x in]
# The GEMVs of one 7B-shape decode step: (rows, cols, launches per step) -- fused q|k|v, wo, the
# row-interleaved w1|w3, w2, and the classifier.
DECODE_GEMVS = [(12288, 4096, 32), (4096, 4096, 32), (22016, 4096, 32), (4096, 11008, 32), (32000, 4096, 1)]
# DRAM bytes / algorithmic bytes of one batched GEMV launch, from the ncu capture of every bench shape
# summarised in profiles/gemv_q8_batch.txt (dram__bytes_read.sum + dram__bytes_write.sum: 0.995-1.004
# for the 4096- and 11008-row shapes).
NCU_GEMV_TRAFFIC_RATIO = 1.000
# DRAM bytes / algorithmic bytes of one persistent decode-step launch (step_kernel), from the ncu
# capture summarised in profiles/step_kernel_7b.txt (full 7B shape, positions 40-43).
NCU_STEP_TRAFFIC_RATIO = 1.005


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "gemv", "gemm", "attention"], default="decode")
    ap.add_argument("--kv", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--model", choices=["7b", "70b"], default="7b",
                    help="7b: the headline workload; 70b: the 70B-shape GQA model, 512-token prompt, 128 tokens")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the long-prompt prefill and GEMM measurements")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the long-context (2048-token prompt) and 70B-shape measurements")
    ap.add_argument("--layers", type=int, default=0,
                    help="truncate the 7B shape to this many layers (a small case of the same kernel, for profiling)")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks during the timed region
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index  # an index, or a comma-separated list of indices
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------ model construction on the GPU
def weight_bytes_per_token(cfg) -> float:
    """Algorithmic bytes a decode step reads: every matmul weight at 1.125 B per value (int8 + fp32
    scale per 32), the activation vectors, one embedding row, the norm weights."""
    mats = [(cfg.dim, cfg.dim), (cfg.kv_dim, cfg.dim), (cfg.kv_dim, cfg.dim), (cfg.dim, cfg.dim),
            (cfg.hidden_dim, cfg.dim), (cfg.dim, cfg.hidden_dim), (cfg.hidden_dim, cfg.dim)]
    per_layer = sum(d * n * 1.125 + n * 1.125 + d * 4 for d, n in mats) + 2 * cfg.dim * 4
    cls = cfg.vocab_size * cfg.dim * 1.125 + cfg.dim * 1.125 + cfg.vocab_size * 4
    return cfg.n_layers * per_layer + cls + cfg.dim * 1.125 + cfg.dim * 4


def kv_bytes_read(cfg, pos0: int, pos1: int, elem: int) -> float:
    """KV-cache bytes the attention reads over positions [pos0, pos1): 2 * (pos+1) * kv_dim per layer."""
    tot = sum(pos + 1 for pos in range(pos0, pos1))
    return 2.0 * tot * cfg.kv_dim * elem * cfg.n_layers


def build_model(cfg, kv_f32: bool, seed: int, rank: int = 0, world: int = 1, device: int = 0):
    """The synthetic model on this GPU (this rank's shard of it under tensor parallelism): every rank
    generates the same full weights on its GPU from the seed and the engine keeps its slices."""
    import torch

    from diolkos_b200 import ops, synth, tp
    from diolkos_b200.model import Model, weight_id

    m = Model(cfg, kv_f32=kv_f32, device=device, tp_rank=rank, tp_world=world)
    g = torch.Generator(device="cuda")
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        which, layer = weight_id(name)
        n = 1
        for s in shape:
            n *= s
        if kind == "norm":
            m.set_weight_device(which, layer, torch.ones(n, device="cuda", dtype=torch.float32))
            continue
        g.manual_seed(seed * 1000003 + idx)
        w = (torch.randn(n, generator=g, device="cuda", dtype=torch.float32) * 0.02).to(torch.bfloat16)
        q, s = ops.quantize_bf16(w.view(torch.int16))
        del w
        torch.cuda.synchronize()
        m.set_weight_device(which, layer, q, s)
        del q, s
    if world > 1:
        tp.connect(m)
    m.finalize()
    return m


# ------------------------------------------------------------------ CPU baseline: the reference
def physical_cores() -> int:
    """Physical cores of this host (the reference's OpenMP loops run one thread per core)."""
    try:
        import psutil

        n = psutil.cpu_count(logical=False)
        if n:
            return int(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def host_weights(cfg, seed: int, device: int = 0):
    """The seeded weights of build_model, tensor by tensor, brought to the host: (name, kind, value) with
    value = (int8 q, fp32 s) planar Q8_0 or an fp32 vector.  Generated on the GPU from the same seeds and
    quantised by the library's quantiser, which is bit-exact with the reference loader's
    (convert_bf16_q8_0), so both arms run the same model."""
    import torch

    from diolkos_b200 import ops, synth

    g = torch.Generator(device=f"cuda:{device}")
    for idx, (name, kind, shape) in enumerate(synth.tensor_specs(cfg)):
        n = 1
        for d in shape:
            n *= d
        if kind == "norm":
            yield name, kind, np.ones(n, np.float32)
            continue
        g.manual_seed(seed * 1000003 + idx)
        with torch.cuda.device(device):
            w = (torch.randn(n, generator=g, device=f"cuda:{device}", dtype=torch.float32) * 0.02).to(torch.bfloat16)
            q, sc = ops.quantize_bf16(w.view(torch.int16))
            torch.cuda.synchronize()
            yield name, kind, (q.cpu().numpy(), sc.cpu().numpy())
            del w, q, sc


def write_reference_model(root: str, cfg, seed: int, name: str = "llama7b") -> str:
    """The model directory the reference loads: config.json, a header-only safetensors and the Q8_0 / F32
    cache files its loader reads instead of quantising (src/safetensors.c:57-114), written from
    host_weights.  Returns the model directory (its cache sits in root/cache/<name>)."""
    from diolkos_b200 import synth

    md = os.path.join(root, name)
    synth.write_model(md, cfg, seed, header_only=True)
    cache = os.path.join(root, "cache", name)
    for tname, kind, val in host_weights(cfg, seed):
        if kind == "q8":
            synth.write_q8_cache(cache, tname, val[0], val[1])
        else:
            synth.write_f32_cache(cache, tname, val)
    return md


class CpuReference:
    """The reference's own generate loop on the host cores: its unmodified sources compiled with its own
    flags (oracle/_ref, -march=native build) driven through ref_driver.c (oref_generate: the loop of
    src/bin/localinfer.c:42-99 on token ids), loading the decode workload's model -- the same weights as
    the GPU arm -- from Q8_0 cache files, all physical cores.  Where the reference build is absent, the
    restatement (oracle/port.c) runs the same loop."""

    def __init__(self, cfg, seed: int = None):
        seed = SEED if seed is None else seed
        from oracle import Ref, ref_path

        self.cfg = cfg
        self.want = physical_cores()
        self.tmp = tempfile.mkdtemp(prefix="dk_cpu_")
        self.kind = "reference" if ref_path("native") or ref_path() else "port"
        if self.kind == "reference":
            self.variant = "native" if ref_path("native") else "portable"
            ref = Ref(self.variant)
            self.cores = ref.threads(self.want)  # overrides a launcher's OMP_NUM_THREADS=1
            md = write_reference_model(self.tmp, cfg, seed)
            self.m = ref.load(md, self.tmp)
        else:
            os.environ["OMP_NUM_THREADS"] = str(self.want)
            self.variant = "port"
            self.cores = self.want
            self.m = port_model(cfg, seed)

    def generate(self, prompt, steps):
        """(generated tokens, seconds of the positions that produced them, top-2 logits per token)."""
        if self.kind == "reference":
            return self.m.generate_timed(prompt, steps)
        n_prompt = len(prompt)
        t0 = time.perf_counter()
        self.m.generate(prompt, n_prompt - 1)  # the forced positions alone
        t1 = time.perf_counter()
        toks = self.m.generate(prompt, steps)
        t2 = time.perf_counter()
        return toks, (t2 - t1) - (t1 - t0), None

    def close(self):
        """Drop the model files (the reference keeps its weights mapped from them until exit; fine on Linux)."""
        import shutil

        shutil.rmtree(self.tmp, ignore_errors=True)

    def warm(self, prompt):
        """Page the weights in: a few positions of the loop."""
        self.generate(prompt, min(len(prompt), 4))

    def describe(self, P, G) -> str:
        return (f"{'oracle/_ref (the reference built with its own flags, -march=' + self.variant + ')' if self.kind == 'reference' else 'oracle/port.c restatement'}: "
                f"its generate loop over the {self.cfg.n_layers}-layer model with the GPU arm's weights, {P}-token "
                f"prompt forced one position at a time, then {G} greedy tokens; tok/s = generated tokens / wall "
                f"time of the positions that produced them; bf16 KV (the reference's); {self.cores} OpenMP threads "
                f"({self.want} physical cores)")


def port_model(cfg, seed: int, kv_f32: bool = False):
    """The oracle's restatement (oracle/port.c) loaded with the decode workload's weights (bf16 KV, the
    reference's cache type, unless kv_f32)."""
    from oracle import Port, PortModel

    from diolkos_b200.model import weight_id

    w = {}
    for tname, kind, val in host_weights(cfg, seed):
        w[(_port_key(weight_id(tname)[0]), weight_id(tname)[1])] = val
    return PortModel(Port(), cfg, w, kv_f32=kv_f32)


def _port_key(which: int) -> int:
    import oracle
    from diolkos_b200 import _native as N

    return {N.DK_W_EMB: oracle.PW_EMB, N.DK_W_RMS_FINAL: oracle.PW_RMS_FINAL, N.DK_W_WCLS: oracle.PW_WCLS,
            N.DK_W_RMS_ATT: oracle.PW_RMS_ATT, N.DK_W_WQ: oracle.PW_WQ, N.DK_W_WK: oracle.PW_WK,
            N.DK_W_WV: oracle.PW_WV, N.DK_W_WO: oracle.PW_WO, N.DK_W_RMS_FFN: oracle.PW_RMS_FFN,
            N.DK_W_W1: oracle.PW_W1, N.DK_W_W2: oracle.PW_W2, N.DK_W_W3: oracle.PW_W3}[which]


# The reference's greedy stream of the decode workload (tests/golden/make_llama7b_stream.py: oracle/_ref
# portable build, the GPU arm's weights): the check for runs that do not run the reference themselves.
STREAM_FIXTURE = os.path.join(ROOT, "tests", "golden", "llama7b_greedy.json")


def token_check(gpu_toks, ref_toks, ref_top2, source: str) -> dict:
    """Greedy tokens of the GPU arm against a reference stream: identical count, first divergence and the
    reference's top-2 logit gap there (relative to the top logit; a near-tie when small)."""
    gpu_toks = [int(t) for t in gpu_toks]
    ref_toks = [int(t) for t in ref_toks]
    n = min(len(gpu_toks), len(ref_toks))
    first = next((i for i in range(n) if gpu_toks[i] != ref_toks[i]), None)
    out = {"identical": n if first is None else first, "of": n, "first_divergence": first, "vs": source}
    if first is not None and ref_top2 is not None and first < len(ref_top2):
        a, b = float(ref_top2[first][0]), float(ref_top2[first][1])
        out["ref_top2_gap_at_divergence"] = round((a - b) / abs(a), 7) if a else None
    return out


# ------------------------------------------------------------------ GEMV microbenchmark (config 2)
def forced_check(m, prompt, ref_toks, ref_top2, world: int, source: str) -> dict:
    """Teacher-forced agreement with a reference stream: the model is fed the prompt and then the
    reference's own tokens, and at every generated position its greedy choice (the first index of the
    largest logit, over all ranks' classifier rows) is compared with the reference's.  A free-running
    stream diverges for good at its first near-tie; this count shows whether every disagreement is one.
    Each disagreement lists the reference's top-2 gap and the model's own gap between its choice and the
    reference's token (both relative to the top logit).  Every rank calls it (forward exchanges)."""
    import torch.distributed as dist

    P = len(prompt)
    seq = [int(t) for t in prompt] + [int(t) for t in ref_toks]
    local = []  # per generated position: (best value, best global index, value of the reference's token)
    for pos in range(P - 1 + len(ref_toks)):
        lg = m.forward(seq[pos], pos)
        if pos < P - 1:
            continue
        ok = np.isfinite(lg)  # tensor parallel: this rank's classifier rows
        idx = np.flatnonzero(ok)
        b = int(idx[np.argmax(lg[idx])])
        rt = seq[pos + 1]
        local.append((float(lg[b]), b, float(lg[rt]) if ok[rt] else float("nan")))
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, local)
    else:
        allr = [local]
    agree, dis = 0, []
    for j in range(len(ref_toks)):
        cands = [r[j] for r in allr]
        top = max(c[0] for c in cands)
        best = min(c[1] for c in cands if c[0] == top)
        rv = next(c[2] for c in cands if c[2] == c[2])
        if best == int(ref_toks[j]):
            agree += 1
            continue
        d = {"index": j, "gpu": best, "ref": int(ref_toks[j]), "gpu_gap": round((top - rv) / abs(top), 7)}
        if ref_top2 is not None and j < len(ref_top2):
            a, b2 = float(ref_top2[j][0]), float(ref_top2[j][1])
            d["ref_top2_gap"] = round((a - b2) / abs(a), 7) if a else None
        dis.append(d)
    return {"agree": agree, "of": len(ref_toks), "vs": source,
            "max_gap_at_disagreement": max((max(d["gpu_gap"], d.get("ref_top2_gap") or 0.0) for d in dis), default=None),
            "disagreements": dis[:16]}


def gemv_alg_bytes(d: int, n: int) -> float:
    """Algorithmic bytes of one [d x n] Q8_0 GEMV: weights + scales, the activation, the output."""
    return d * n * 1.125 + n * 1.125 + d * 4


def graph_time_us(enqueue, calls: int, reps: int = 10) -> float:
    """Device time per call of `enqueue` (which issues `calls` library calls on torch's current stream),
    captured once in a CUDA graph so that host launch overhead is not timed: `reps` replays back to back,
    each between its own pair of CUDA events, behind one untimed replay that keeps the stream busy while
    the host enqueues the rest; the median replay over `calls`."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        enqueue()  # outside capture: any first-call setup of the library happens here
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    # thread_local: CUDA calls of other threads (a process group's watchdog under torchrun) stay legal
    # while this thread captures
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        enqueue()
    graph.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    graph.replay()
    for e0, e1 in ev:
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    del graph
    times = sorted(e0.elapsed_time(e1) * 1e3 / calls for e0, e1 in ev)
    return times[len(times) // 2]


def gemv_bench(reps: int = 64, shapes=None):
    """GEMV shapes through dk_matmul_q8_0_batch: `reps` GEMVs in one call, rotating over enough
    packed copies of the matrix that the working set is over 3x the L2; device time per GEMV
    (graph_time_us: CUDA graph, CUDA events on the launching stream, median of 10 replays)."""
    import torch

    from diolkos_b200 import ops

    out = {}
    for d, n in (shapes or GEMV_SHAPES):
        copies = max(2, int(3 * 126e6 // ops.packed_bytes(n, d)) + 1)
        g = torch.Generator(device="cuda").manual_seed(d * 31 + n)
        ws = []
        for _ in range(copies):
            wf = (torch.randn(d * n, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            q, s = ops.quantize_bf16(wf.view(torch.int16))
            ws.append(ops.pack(q, s, n, d))
            del wf, q, s
        x = torch.randn(n, generator=g, device="cuda")
        batch = [ws[i % copies] for i in range(reps)]
        y = torch.empty((reps, d), device="cuda")
        best = graph_time_us(lambda: ops.matmul_batch(x, batch, n, d, y), reps)
        alg = gemv_alg_bytes(d, n)
        out[f"{d}x{n}"] = {"us": round(best, 2), "GBps": round(alg / best / 1e3, 1)}
        del ws, batch, y
        torch.cuda.empty_cache()
    return out


PREFILL_LEN = 2048  # the long prompt of the tensor-parallel workload, prefilled on one GPU here
GEMM_TOKENS = 256   # positions per prefill chunk (the engine's chunk)


def gemm_ops(cfg, ntok: int) -> float:
    """Int8 multiply-adds (x2) of the prefill matmuls over ntok positions: q|k|v, wo, w1|w3, w2."""
    per_layer = cfg.dim * (cfg.dim + 2 * cfg.kv_dim) + cfg.dim * cfg.dim + 2 * cfg.hidden_dim * cfg.dim + cfg.dim * cfg.hidden_dim
    return 2.0 * per_layer * cfg.n_layers * ntok


def int8_peak():
    """Dense int8 tensor peak: twice the measured bf16 cuBLAS burst (B200's int8 rate is 2x bf16)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return 2.0 * float(json.load(f)["bf16_tflops"]), "2 x measured bf16 burst"
    except Exception:
        return 2.0 * 1590.0, "2 x fallback bf16"


def prefill_bench(m, cfg, reps: int = 3):
    """The batched prefill of a PREFILL_LEN-token seeded prompt (dk_model_prefill, positions
    0..PREFILL_LEN-1, chunks of 256), CUDA events on the engine's stream, best of `reps`."""
    import torch

    from diolkos_b200 import synth

    L = min(PREFILL_LEN, cfg.seq_len)
    prompt = synth.seeded_prompt(SEED + 1, L, cfg.vocab_size)
    stream = torch.cuda.ExternalStream(m.stream)
    m.set_tokens(prompt, n_forced=L)
    m.prefill(0, L)  # warm-up (allocates the chunk scratch)
    m.sync()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.prefill(0, L)
        e1.record(stream)
        m.sync()
        best = min(best, e0.elapsed_time(e1))
    if m.device_error():
        raise RuntimeError("device error word after the prefill")
    ops = gemm_ops(cfg, L)
    return {"positions": L, "ms": round(best, 3), "tok_per_s": round(L / (best / 1e3), 1),
            "int8_tops": round(ops / (best / 1e3) / 1e12, 1),
            "what": "dk_model_prefill of a seeded prompt, all layers (matmuls, attention over the growing "
                    "KV cache, activations), CUDA events; int8_tops = matmul multiply-adds x2 / time"}


def gemm_bench(cfg, ntok: int = GEMM_TOKENS, reps: int = 8):
    """The prefill matmul (dk_matmul_q8_0_tokens) on one layer's shapes at ntok positions: reps
    launches back to back rotating over packed copies (working set > 3x L2), behind one untimed launch
    so that the first timed one does not wait for the host; CUDA events, best of 3."""
    import torch

    from diolkos_b200 import ops

    shapes = [(cfg.dim + 2 * cfg.kv_dim, cfg.dim), (cfg.dim, cfg.dim), (2 * cfg.hidden_dim, cfg.dim),
              (cfg.dim, cfg.hidden_dim)]
    out, tot_ops, tot_us = {}, 0.0, 0.0
    for d, n in shapes:
        copies = max(2, int(3 * 126e6 // ops.packed_bytes(n, d)) + 1)
        g = torch.Generator(device="cuda").manual_seed(d * 17 + n)
        ws = []
        for _ in range(copies):
            wf = (torch.randn(d * n, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
            q, s = ops.quantize_bf16(wf.view(torch.int16))
            ws.append(ops.pack(q, s, n, d))
            del wf, q, s
        xf = torch.randn(ntok * n, generator=g, device="cuda").to(torch.bfloat16)
        xq, xs = ops.quantize_bf16(xf.view(torch.int16))
        xq, xs = xq.view(ntok, n), xs.view(ntok, n // 32)
        y = torch.empty((ntok, d), device="cuda")
        ops.matmul_tokens(xq, xs, ws[0], n, d, out=y)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ops.matmul_tokens(xq, xs, ws[copies - 1], n, d, out=y)  # the stream is busy when e0 is reached
            e0.record()
            for i in range(reps):
                ops.matmul_tokens(xq, xs, ws[i % copies], n, d, out=y)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e3 / reps)
        o = 2.0 * d * n * ntok
        tot_ops += o
        tot_us += best
        out[f"{d}x{n}"] = {"us": round(best, 2), "int8_tops": round(o / best / 1e6, 1)}
        del ws, y, xq, xs
        torch.cuda.empty_cache()
    peak, kind = int8_peak()
    ach = tot_ops / tot_us / 1e6
    return {"tokens": ntok, "shapes": out, "achieved_tops": round(ach, 1), "peak_tops": round(peak, 1),
            "frac": round(ach / peak, 4), "peak_kind": kind, "kernel": "gemm_q8_tma_kernel",
            "what": "one layer's four prefill matmuls at 256 positions (the engine's chunk), int8 multiply-adds x2 "
                    "/ CUDA-event time per launch"}


# ------------------------------------------------------------------ main arms
def workload_config(cfg, model_name, P, G, kv: str, world: int, layers_note: str = "") -> dict:
    """The `config` object both arms print for the decode workload."""
    return {"workload": f"{model_name} q8_0 decode: {P}-token prompt, then {G} greedy tokens timed" + layers_note,
            "model": model_name, "dim": cfg.dim, "hidden": cfg.hidden_dim, "layers": cfg.n_layers,
            "heads": cfg.n_heads, "kv_heads": cfg.n_kv_heads, "vocab": cfg.vocab_size, "seq_len": cfg.seq_len,
            "kv_cache": kv, "global_batch": 1,
            "parallelism": "single GPU" if world == 1 else
            f"tp{world}: heads / w1,w3 rows / classifier rows per GPU, wo and w2 partial sums exchanged inside "
            f"the GEMVs over NVLink peer memory",
            "l2": f"weights ({weight_bytes_per_token(cfg) / 1e9:.1f} GB) exceed L2; every token streams them from HBM"}


# Wall-clock budget of the reference arm's timed steps: each step is the whole workload (tens of seconds on a
# CPU); steps past the budget are not run, and the line says how many ran.
REFERENCE_BUDGET_S = 150.0


def run_reference(args):
    """The reference arm: the reference's own generate loop (CpuReference) over the decode workload, each
    timed step one full run of it (32-token prompt forced one position at a time, 256 greedy tokens)."""
    from diolkos_b200 import synth

    cfg, P, G, model_name = _models()["7b"]
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))  # only to generate the seeded weights
    cpu = CpuReference(cfg)
    prompt = synth.seeded_prompt(SEED, P, cfg.vocab_size)
    for _ in range(args.warmup):
        cpu.warm(prompt)
    n_tok, secs, runs = 0, 0.0, 0
    toks = None
    t_start = time.perf_counter()
    for _ in range(args.steps):
        toks, gs, _ = cpu.generate(prompt, P - 1 + G)
        n_tok += len(toks)
        secs += gs
        runs += 1
        if time.perf_counter() - t_start > REFERENCE_BUDGET_S:
            break
    cpu.close()
    v = n_tok / secs
    kv = "bf16 (the reference has no fp32 cache)"
    line = {
        "impl": "reference", "metric": "Q8_0 decode tok/s batch 1", "value": round(v, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "steps_run": runs, "warmup": args.warmup,
        "ms_per_step": round(1e3 * secs / runs, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,0.02) weights, seeded prompt)",
        "config": workload_config(cfg, model_name, P, G, kv, args.gpus),
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": cpu.cores, "kind": cpu.kind,
                         "sample": cpu.describe(P, G) + f"; {runs} full run(s) of the workload"},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "tokens_sample": [int(t) for t in toks[:8]],
    }
    print(json.dumps(line), flush=True)
    return 0


LONG_PROMPT = 2048  # config 4: the long prompt, prefilled on the tensor cores, then GEN_LEN decode tokens


def decode_roofline(cfg, P, G, ms_per_tok, world, kv_f32) -> dict:
    """Weight + KV bytes per token over the decode positions P-1 .. P-2+G, per rank, against the HBM peak."""
    elem = 4 if kv_f32 else 2
    bytes_tok = weight_bytes_per_token(cfg) + kv_bytes_read(cfg, P - 1, P - 1 + G, elem) / G
    hbm, kind = peaks()
    rank_gbps = bytes_tok / world / (ms_per_tok / 1e3) / 1e9
    return {"bound": "hbm", "achieved": round(rank_gbps, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(rank_gbps / hbm, 4), "bytes_per_token_per_rank": round(bytes_tok / world),
            "what": f"weight + KV bytes per token per rank / time per token; peak = {kind} HBM copy bandwidth"}


def run_decode(args):
    import torch

    from diolkos_b200 import synth, tp

    cfg, P, G, model_name = _models()[args.model]
    if args.layers > 0:
        cfg = cfg.replace(n_layers=args.layers)
    kv_f32 = args.kv == "f32"
    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        if int(os.environ.get("WORLD_SIZE", "1")) != world:
            raise RuntimeError(f"--gpus {world} needs {world} ranks (torchrun --nproc-per-node {world})")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def check_err(m, what):
        err = int(max_over_ranks(float(m.device_error())))  # every rank takes the same exit
        if err:
            raise RuntimeError(f"device error word 0x{err:x} {what}")

    m = build_model(cfg, kv_f32, SEED, rank, world, local)
    stream = torch.cuda.ExternalStream(m.stream)
    prompt = synth.seeded_prompt(SEED, P, cfg.vocab_size)

    def one_step(mm, pr, g, record=None):
        mm.set_tokens(pr, n_forced=len(pr))
        if record:
            record[2].record(stream_of[id(mm)])
        mm.prefill(0, len(pr) - 1)  # the forced prompt positions on the tensor cores
        if record:
            record[0].record(stream_of[id(mm)])
        mm.enqueue_steps(len(pr) - 1, g)
        if record:
            record[1].record(stream_of[id(mm)])

    stream_of = {id(m): stream}

    def timed_decode(mm, pr, g, steps, warmup):
        """warm-up, then `steps` timed runs of prefill + g greedy tokens: (decode ms, prompt ms per run)."""
        torch.cuda.synchronize()
        barrier()
        for _ in range(warmup):
            one_step(mm, pr, g)
        mm.sync()
        check_err(mm, "after warm-up")
        torch.cuda.synchronize()
        barrier()
        evs = []
        for _ in range(steps):
            e = tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
            one_step(mm, pr, g, e)
            evs.append(e)
        mm.sync()
        torch.cuda.synchronize()
        barrier()
        dec = max_over_ranks(sum(a.elapsed_time(b) for a, b, _ in evs))
        pro = max_over_ranks(sum(c.elapsed_time(a) for a, _, c in evs)) / steps
        check_err(mm, "after the timed runs")
        return dec, pro

    # ---- headline: the decode workload (config 3 at N = 1, its tensor-parallel split at N > 1)
    sampler = ClockSampler(",".join(str(i) for i in range(world)) if rank == 0 else local)
    # the ranks start together: the prefill's and the decode step's cross-rank waits are bounded
    torch.cuda.synchronize()
    barrier()
    for _ in range(args.warmup):
        one_step(m, prompt, G)
    m.sync()
    check_err(m, "after warm-up")
    if rank == 0:
        sampler.start()
    torch.cuda.synchronize()
    m.sync()
    barrier()
    t_all0 = time.perf_counter()
    evs = []
    for _ in range(args.steps):
        e = tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
        one_step(m, prompt, G, e)
        evs.append(e)
    m.sync()
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - t_all0
    clocks = sampler.stop() if rank == 0 else None
    decode_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b, _ in evs))
    prompt_ms = max_over_ranks(sum(c.elapsed_time(a) for a, _, c in evs)) / args.steps
    check_err(m, "after the timed steps")
    toks = m.get_tokens(P + G)

    value = G * args.steps / (decode_ms / 1e3)
    ms_per_tok = decode_ms / (G * args.steps)
    elem = 4 if kv_f32 else 2
    bytes_tok = weight_bytes_per_token(cfg) + kv_bytes_read(cfg, P - 1, P - 1 + G, elem) / G
    hbm, peak_kind = peaks()
    achieved = bytes_tok / (ms_per_tok / 1e3) / 1e9
    rank_bytes = bytes_tok / world  # every rank streams its shard of the weights and KV heads
    step_gbps = rank_bytes / (ms_per_tok / 1e3) / 1e9

    # end to end through the public C-ABI generate entry point (host buffers)
    e2e_times = []
    n_gen = 0
    for _ in range(max(1, args.steps)):
        barrier()
        t0 = time.perf_counter()
        gen = m.generate(prompt, P - 1 + G)
        e2e_times.append(max_over_ranks(time.perf_counter() - t0))
        n_gen = len(gen)
    e2e = n_gen * len(e2e_times) / sum(e2e_times)
    kernels_per_step = m.kernels_per_step

    # ---- config 4: 2048-token prompt prefilled on the tensor cores, then 256 tokens at long context
    long_ctx = None
    if args.model == "7b" and not args.no_extra and not args.layers:
        Lp = min(LONG_PROMPT, cfg.seq_len - G)
        lprompt = synth.seeded_prompt(SEED + 1, Lp, cfg.vocab_size)
        s2 = ClockSampler(",".join(str(i) for i in range(world)) if rank == 0 else local)
        if rank == 0:
            s2.start()
        dec, pro = timed_decode(m, lprompt, G, 2, 1)
        c2 = s2.stop() if rank == 0 else None
        mt = dec / (2 * G)
        long_ctx = {"workload": f"llama2-7b-shape: {Lp}-token seeded prompt, its {Lp - 1} forced positions prefilled "
                                f"(int8 tensor-core matmuls{', tensor parallel' if world > 1 else ''}), then {G} greedy "
                                f"tokens at positions {Lp - 1}..{Lp - 2 + G}",
                    "value": round(1e3 / mt, 2), "unit": "tok/s", "ms_per_token": round(mt, 4),
                    "prefill_ms": round(pro, 3), "prefill_positions_per_s": round((Lp - 1) / (pro / 1e3), 1),
                    "roofline": decode_roofline(cfg, Lp, G, mt, world, kv_f32), "steps": 2, "warmup": 1,
                    "clocks": c2}

    long_prefill = prefill_bench(m, cfg) if world == 1 and not args.no_prefill else None
    m.close()  # every rank leaves the exchange at the same point
    barrier()

    # ---- the greedy stream with the reference's cache type (bf16 KV), for the token check against it, and
    # the same model teacher-forced with the reference's stream
    bf16_toks, forced = None, None
    fx = None
    if args.model == "7b" and not args.layers and os.path.exists(STREAM_FIXTURE):
        with open(STREAM_FIXTURE) as f:
            fx = json.load(f)
        if not (fx.get("seed") == SEED and fx.get("prompt") == [int(t) for t in prompt]):
            fx = None
    if args.model == "7b" and not args.layers:
        mb = build_model(cfg, False, SEED, rank, world, local)
        barrier()
        bf16_toks = [int(t) for t in mb.generate(prompt, P - 1 + G)]
        check_err(mb, "after the bf16-KV generate")
        if fx is not None:
            forced = forced_check(mb, prompt, fx["tokens"], fx.get("top2"), world,
                                  f"{os.path.relpath(STREAM_FIXTURE, ROOT)} ({fx.get('reference')})")
            check_err(mb, "after the teacher-forced check")
        mb.close()
        barrier()

    # ---- config 5: the 70B-shape GQA model, 512-token prompt, 128 greedy tokens
    big = None
    if args.model == "7b" and not args.no_extra and not args.layers:
        c70, P70, G70, name70 = _models()["70b"]
        m70 = build_model(c70, kv_f32, SEED, rank, world, local)
        stream_of[id(m70)] = torch.cuda.ExternalStream(m70.stream)
        pr70 = synth.seeded_prompt(SEED, P70, c70.vocab_size)
        s3 = ClockSampler(",".join(str(i) for i in range(world)) if rank == 0 else local)
        if rank == 0:
            s3.start()
        dec, pro = timed_decode(m70, pr70, G70, 2, 1)
        c3 = s3.stop() if rank == 0 else None
        mt = dec / (2 * G70)
        big = {"workload": f"{name70} (dim {c70.dim}, hidden {c70.hidden_dim}, {c70.n_layers} layers, {c70.n_heads} "
                           f"heads over {c70.n_kv_heads} KV heads): {P70}-token prompt prefilled, then {G70} greedy "
                           f"tokens", "value": round(1e3 / mt, 2), "unit": "tok/s", "ms_per_token": round(mt, 4),
               "prefill_ms": round(pro, 3), "roofline": decode_roofline(c70, P70, G70, mt, world, kv_f32),
               "weight_gb": round(weight_bytes_per_token(c70) / 1e9, 2), "steps": 2, "warmup": 1, "clocks": c3}
        m70.close()
        barrier()

    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    # The dominant kernel's companion: the GEMV over this rank's shapes and launch counts of one decode step.
    sh = tp.shard(cfg, rank, world)
    ld, lkv, lh = sh.q_rows[1] - sh.q_rows[0], sh.kv_rows[1] - sh.kv_rows[0], sh.hidden_rows[1] - sh.hidden_rows[0]
    lv = sh.vocab_rows[1] - sh.vocab_rows[0]
    decode_gemvs = [(ld + 2 * lkv, cfg.dim, cfg.n_layers), (cfg.dim, ld, cfg.n_layers),
                    (2 * lh, cfg.dim, cfg.n_layers), (cfg.dim, lh, cfg.n_layers), (lv, cfg.dim, 1)]
    gemv = gemv_bench() if world == 1 else None
    gemm = gemm_bench(cfg) if world == 1 and not args.no_prefill else None
    mix = gemv_bench(shapes=[(d, n) for d, n, _ in decode_gemvs])
    mix_bytes = sum(c * gemv_alg_bytes(d, n) for d, n, c in decode_gemvs)
    mix_us = sum(c * mix[f"{d}x{n}"]["us"] for d, n, c in decode_gemvs)
    launches = sum(c for _, _, c in decode_gemvs)
    gemv_gbps = mix_bytes / mix_us / 1e3

    # ---- the reference on the host cores (N = 1): one full run of the workload; its greedy stream
    cpu, checks = None, {}
    gpu_toks = [int(t) for t in toks[P:P + G]]
    cmp_toks = bf16_toks if bf16_toks is not None else gpu_toks
    if not args.no_cpu_baseline and world == 1 and args.model == "7b" and not args.layers:
        try:
            cb = CpuReference(cfg)
            cb.warm(prompt)
            rt, secs, top2 = cb.generate(prompt, P - 1 + G)
            v = len(rt) / secs
            cpu = {"value": round(v, 3), "unit": "tok/s", "cores": cb.cores, "kind": cb.kind,
                   "sample": cb.describe(P, G) + "; one full run of the workload"}
            checks["this_run"] = token_check(cmp_toks, rt, top2, f"this run's {cb.kind} ({cb.variant} build)")
            cb.close()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": physical_cores(), "kind": "reference",
                   "sample": f"not run: {ex}"}
    if fx is not None:
        checks["fixture"] = token_check(cmp_toks, fx["tokens"], fx.get("top2"),
                                        f"{os.path.relpath(STREAM_FIXTURE, ROOT)} ({fx.get('reference')})")
    if forced is not None:
        if fx.get("control_forced"):
            c = fx["control_forced"]
            forced["control"] = {k: c.get(k) for k in ("what", "agree", "of", "max_gap_at_disagreement")}
        checks["forced"] = forced
    if bf16_toks is not None:
        checks["gpu_stream"] = ("greedy tokens of the same model with the reference's bf16 KV cache (dk_model_generate), "
                                "compared with the reference's stream; the headline decode uses an fp32 cache, "
                                f"whose stream agrees with the bf16 one for {token_check(gpu_toks, bf16_toks, None, '')['identical']} "
                                f"of {G} tokens")

    line = {
        "metric": "Q8_0 decode tok/s batch 1", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(decode_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,0.02) weights, seeded prompt)",
        "config": workload_config(cfg, model_name, P, G, args.kv, world,
                                  f" ({cfg.n_layers} layers: profiling case)" if args.layers else ""),
        "ms_per_token": round(ms_per_tok, 4),
        # the prefill launches per chunk 10 kernels per layer (activation, matmul, KV write, attention, then
        # activation + matmul for wo, w1|w3, w2; tensor parallel: + scatter, signal, wait, reduce after wo
        # and after w2) and 3 for the last layer (its K/V rows); then one persistent step per token
        "gpu_launches": (kernels_per_step * G + ((cfg.n_layers - 1) * (10 + (8 if world > 1 else 0)) + 3) *
                         (-(-(P - 1) // GEMM_TOKENS))) * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(step_gbps, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(step_gbps / hbm, 4),
                     "traffic": (round(NCU_STEP_TRAFFIC_RATIO * rank_bytes) if NCU_STEP_TRAFFIC_RATIO else None),
                     "kernel": "step_kernel",
                     "what": f"the persistent decode step (one launch per token, {kernels_per_step} kernel per step): "
                             f"this rank's weight + KV bytes per token ({rank_bytes / 1e9:.3f} GB) / time per token "
                             f"(CUDA events around back-to-back steps); peak = {peak_kind} HBM copy bandwidth; "
                             f"traffic = DRAM bytes per launch"},
        "gemv_roofline": {"bound": "hbm", "achieved": round(gemv_gbps, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(gemv_gbps / hbm, 4),
                          "traffic": (round(NCU_GEMV_TRAFFIC_RATIO * mix_bytes / launches)
                                      if NCU_GEMV_TRAFFIC_RATIO else None),
                          "kernel": "gemv_q8_kernel",
                          "what": f"Q8_0 GEMV over one decode step's {launches} launches on rank 0 (shapes "
                                  f"{decode_gemvs}): {mix_bytes / launches / 1e6:.2f} MB algorithmic bytes per launch / "
                                  f"{mix_us / launches:.2f} us average launch (CUDA events, back-to-back batches); "
                                  f"peak = {peak_kind} HBM copy bandwidth; traffic = DRAM bytes per launch"},
        "step_roofline": {"achieved": round(achieved, 1), "frac": round(achieved / (hbm * world), 4),
                          "unit": "GB/s",
                          "what": f"whole decode step: weight + KV bytes per token ({bytes_tok / 1e9:.3f} GB) / "
                                  f"time per token, against {world} x the HBM peak"},
        "tokens_check": checks or None,
        "long_context": long_ctx,
        "llama70b": big,
        "gemv": gemv,
        "gemv_decode_shapes": mix,
        "prompt_prefill_ms": round(prompt_ms, 3),
        "prefill": long_prefill,
        "prefill_gemm": gemm,
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * P + 12,
                "d2h_bytes_per_step": 4 * (P + G) + 4,
                "how": "dk_model_generate (C ABI): host prompt -> host tokens, wall clock, prompt prefill included"},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "wall_s_timed_region": round(wall, 3),
        "tokens_sample": gpu_toks[:8],
    }
    print(json.dumps(line), flush=True)
    return 0


def run_gemv(args):
    import torch

    torch.cuda.set_device(0)
    g = gemv_bench(reps=max(20, args.steps * 10))
    mix = gemv_bench(reps=max(20, args.steps * 10), shapes=[(d, n) for d, n, _ in DECODE_GEMVS])
    hbm, kind = peaks()
    best = max(g.items(), key=lambda kv: kv[1]["GBps"])
    line = {"metric": "Q8_0 GEMV HBM GB/s", "value": best[1]["GBps"], "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "isolated Q8_0 GEMV, batch 1", "shapes": g}, "decode_shapes": mix, "peak": hbm,
            "peak_kind": kind}
    print(json.dumps(line), flush=True)
    return 0


def run_gemm(args):
    """The prefill matmul alone (dk_matmul_q8_0_tokens) on one 7B layer's shapes at 256 tokens."""
    import torch

    from diolkos_b200 import synth

    torch.cuda.set_device(0)
    g = gemm_bench(synth.LLAMA7B)
    line = {"metric": "Q8_0 prefill matmul int8 TOPS", "value": g["achieved_tops"], "unit": "TOPS", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "tensor-core Q8_0 matmul, 7B layer shapes, 256 tokens"}, "prefill_gemm": g}
    print(json.dumps(line), flush=True)
    return 0


ATTN_POSITIONS = (200, 2047, 4000)  # a short context, the long-prompt workload's, near seq_len


def attention_bench(reps: int = 32, kv: str = "f32"):
    """The decode attention kernel alone (dk_attention_decode: RoPE, KV-cache write, split-K softmax.V;
    the per-kernel decode path's attention, the same arithmetic as the persistent step's) at the 7B shape
    (32 heads of 128, seq_len 4096) at a few positions.  At each position the calls rotate over enough
    layers' KV caches that the rows they read are over 3x the L2 (at least `reps` calls); device time
    per call (graph_time_us: CUDA graph, CUDA events, median of 10 replays).  GB/s = the KV bytes a call reads
    (2 * (pos+1) * kv_dim * element size) / time."""
    import torch

    from diolkos_b200 import ops, synth

    cfg = synth.LLAMA7B
    H, KVH, hs, seq = cfg.n_heads, cfg.n_kv_heads, cfg.dim // cfg.n_heads, cfg.seq_len
    esz = 4 if kv == "f32" else 2

    def alg_bytes(pos):
        return 2.0 * (pos + 1) * KVH * hs * esz

    def n_copies(pos):
        return max(2, int(3 * 126e6 // alg_bytes(pos)) + 1)

    copies = max(n_copies(pos) for pos in ATTN_POSITIONS)
    g = torch.Generator(device="cuda").manual_seed(5)
    dt = torch.float32 if kv == "f32" else torch.bfloat16
    ks = [(torch.randn(KVH * seq * hs, generator=g, device="cuda") * 0.5).to(dt) for _ in range(copies)]
    vs = [(torch.randn(KVH * seq * hs, generator=g, device="cuda") * 0.5).to(dt) for _ in range(copies)]
    if kv != "f32":
        ks = [k.view(torch.int16) for k in ks]
        vs = [v.view(torch.int16) for v in vs]
    half = hs // 2
    inv = 1.0 / (10000.0 ** (torch.arange(half, dtype=torch.float64) * 2 / hs))
    ang = torch.arange(seq, dtype=torch.float64)[:, None] * inv[None, :]
    rope = torch.stack([torch.cos(ang), torch.sin(ang)], -1).to(torch.float32).reshape(-1).cuda()
    qkv = torch.randn((H + 2 * KVH) * hs, generator=g, device="cuda")
    work = torch.zeros(ops.attention_work_bytes(H, KVH, hs, seq), dtype=torch.uint8, device="cuda")
    out = torch.empty(H * hs, device="cuda")
    hbm, kind = peaks()
    res = {}
    for pos in ATTN_POSITIONS:
        p = torch.tensor([pos], dtype=torch.int32, device="cuda")
        c = n_copies(pos)
        calls = max(reps, c)

        def enqueue():
            for i in range(calls):
                ops.attention_decode(qkv, rope, ks[i % c], vs[i % c], p, H, KVH, hs, seq, work, out)

        best = graph_time_us(enqueue, calls)
        alg = alg_bytes(pos)
        res[str(pos)] = {"us": round(best, 2), "kv_mb": round(alg / 1e6, 2), "GBps": round(alg / best / 1e3, 1),
                         "frac": round(alg / best / 1e3 / hbm, 4), "calls": calls, "caches": c}
    del ks, vs
    torch.cuda.empty_cache()
    return {"kernel": "attention_kernel", "kv": kv, "positions": res, "peak": hbm, "peak_kind": kind,
            "what": f"dk_attention_decode at 32 heads x 128, seq_len {seq}, {kv} KV cache: KV bytes read per call / "
                    "device time per call (the calls of one position captured in a CUDA graph, rotating over "
                    "enough layers' caches that the rows read exceed 3x the L2; median of 10 replays)"}


def run_attention(args):
    import torch

    torch.cuda.set_device(0)
    a = attention_bench(kv=args.kv)
    best = max(a["positions"].values(), key=lambda v: v["GBps"])
    line = {"metric": "decode attention HBM GB/s", "value": best["GBps"], "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.kv, "data": "synthetic",
            "config": {"workload": "decode attention, LLaMA-2-7B heads, one layer per call"}, "attention": a}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "gemv":
        return run_gemv(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload == "attention":
        return run_attention(args)
    return run_decode(args)


if __name__ == "__main__":
    sys.exit(main())
