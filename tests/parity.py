"""Per-layer parity harness: the GPU decode step against an oracle model, checkpoint by checkpoint.

An oracle model is the hooked reference build (oracle/_ref/*/liboracle_ref_hooked.so: the reference's
unmodified forward() with its rmsnorm / matmul calls recorded, oracle/ref_hooks.c) or the restatement
(oracle/port.c) for cache types the reference has no build for.  Both give, per forward(): the logits,
the residual stream before every rmsnorm (transformer.c:76, :204, :234: the embedding row, then x after
every residual add) and, per layer, the fp32 input and Q8_0 form of the wq, wo, w1 and w2 activations
(:83, :196, :208, :225) and of the classifier's (:237).  The GPU engine records the same checkpoints
(dk_model_dump_enable): per GEMV op of the persistent step its input vector and the Q8_0 activation it
built.

Why activations differ.  The reference re-quantises every matmul input to int8.  Its softmax and SwiGLU
call libmvec's vectorised expf (several ulp from the correctly rounded value on about half of all
inputs) and its sums run in the compiler's AVX2 order; a GPU cannot reproduce those bits, so the fp32
inputs of a quantisation differ by a few ulp, and an element whose value x * (1/scale) lies within that
distance of a .5 boundary rounds to the neighbouring int8.  Such a flip moves that matmul's outputs by
one quantum -- up to ~4e-3 relative at dim 288 -- and everything downstream with it.

What ``synced_run`` measures, per position:
  * state synchronisation: before each GPU step the oracle's own KV-cache rows of the previous positions
    are written into the GPU cache (dk_model_kv_write), so every position starts from the same history;
  * end to end against the oracle: every checkpoint upstream of the step's first int8 difference
    (residual stream, attention output, SwiGLU output, logits) and its relative error; the first
    differing activation's int8 values, each to be a +-1 flip whose oracle value lies between the
    rounding boundary and the GPU's value;
  * op by op, replayed on the restatement from the GPU's OWN inputs (so a flip upstream cannot mask a
    fault): every GEMV + residual add bit-exact (matmul_Q8_0 order); every quantisation of an fp32
    input bit-exact, and of an rmsnorm input equal up to +-1 flips within ULP_SLACK ulps of a rounding
    boundary (the rmsnorm's sum of squares runs in a different order); attention (RoPE, the cache write
    and softmax-weighted sum, in float64 from the GPU's own q|k|v) and SwiGLU within OP_TOL.
"""
from __future__ import annotations

import numpy as np

REL_TOL = 1e-3      # the north-star bar for per-layer activations and logits
OP_TOL = 2e-5       # one op replayed in float64 from the GPU's own inputs (fp32 arithmetic + expf ulps)
ULP_SLACK = 4       # ulps of the pre-rounding value allowed beyond the measured input difference
RMS_ULP_SLACK = 8   # ulps from a rounding boundary for an rmsnorm quantisation flip (see replay_ops)


def rel(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = float(np.max(np.abs(b))) if b.size else 0.0
    return float(np.max(np.abs(a - b))) / den if den > 0 else float(np.max(np.abs(a)) if a.size else 0.0)


def pre_round(x, s):
    """The quantiser's pre-rounding values x * (1/scale), fp32 as the reference computes them."""
    inv = (np.float32(1.0) / np.asarray(s, np.float32)).astype(np.float32)
    return (np.asarray(x, np.float32) * np.repeat(inv, 32)).astype(np.float32)


def op_names(n_layers: int):
    names = []
    for l in range(n_layers):
        names += [f"L{l}.qkv", f"L{l}.wo", f"L{l}.w13", f"L{l}.w2"]
    return names + ["cls"]


def _is_norm_op(k: int, n_layers: int) -> bool:
    return k == 4 * n_layers or k % 4 in (0, 2)


def gpu_xres(acts_g, n_layers: int):
    """The GPU's residual checkpoints in the oracle's order: the inputs of the rmsnorm prologues."""
    xs = []
    for l in range(n_layers):
        xs += [acts_g[4 * l][0], acts_g[4 * l + 2][0]]
    return np.stack(xs + [acts_g[4 * n_layers][0]])


def _flip_ok(qo, qg, vo, vg, extra=0.0):
    """+-1 and the boundary between the two int8 values lies between the two pre-rounding values (within
    ULP_SLACK ulps plus `extra`)."""
    b = 0.5 * (qo + qg)
    ulp = float(np.spacing(np.float32(max(abs(vo), 1.0))))
    return abs(qo - qg) == 1 and abs(vo - b) <= abs(vo - vg) + ULP_SLACK * ulp + extra


def cross_flips(acts_o, acts_g, norm_w, port, n_layers: int):
    """Int8 differences between the oracle's and the GPU's activations, op by op: a list of dicts (op
    index, element, oracle int8, GPU int8, distances of both pre-rounding values from the boundary,
    explained).  The GPU's normalised input of an rmsnorm op is recomputed from its dumped residual
    with the restatement's rmsnorm."""
    names = op_names(n_layers)
    flips = []
    for k, ((ai, aq, asc), (gi, gq, gs)) in enumerate(zip(acts_o, acts_g)):
        d = np.nonzero(aq != gq)[0]
        if d.size == 0:
            continue
        xg = port.rmsnorm(np.ascontiguousarray(gi, np.float32), norm_w[k]) if _is_norm_op(k, n_layers) \
            else np.asarray(gi, np.float32)
        vo, vg = pre_round(ai, asc), pre_round(xg, gs)
        for i in d:
            qo, qg = int(aq[i]), int(gq[i])
            b = 0.5 * (qo + qg)
            flips.append({"op": names[k], "k": k, "index": int(i), "oracle": qo, "gpu": qg,
                          "dist_oracle": abs(float(vo[i]) - b), "dist_gpu": abs(float(vg[i]) - b),
                          "explained": _flip_ok(qo, qg, float(vo[i]), float(vg[i]))})
    return flips


def _mm(port, act, wqs):
    xq, xs = act[1], act[2]
    wq, ws = wqs
    n = xq.size
    return port.matmul_q(xq, xs, wq, ws, n, ws.size * 32 // n)


def _rope(v, cs, n_heads_in_v, hs):
    """HF rotate-half RoPE in the reference's fma form, a' = fma(a, c, -(b*s)), b' = fma(a, s, b*c)
    (exact products in float64, one rounding)."""
    v = np.asarray(v, np.float32).reshape(n_heads_in_v, hs)
    c = cs[0::2].astype(np.float64)
    s = cs[1::2].astype(np.float64)
    a, b = v[:, : hs // 2].astype(np.float64), v[:, hs // 2:].astype(np.float64)
    bs = (b * s).astype(np.float32).astype(np.float64)
    bc = (b * c).astype(np.float32).astype(np.float64)
    out = np.empty_like(v)
    out[:, : hs // 2] = (a * c - bs).astype(np.float32)
    out[:, hs // 2:] = (a * s + bc).astype(np.float32)
    return out.reshape(-1)


def _as_f64(rows):
    rows = np.asarray(rows)
    if rows.dtype == np.uint16:
        return (rows.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return rows.astype(np.float64)


def replay_ops(port, w, cfg, acts_g, logits_g, pos, gpu_rows, hist_rows, norm_w, kv_f32: bool):
    """Every op of the GPU step replayed on the restatement from the GPU's own inputs.  gpu_rows(l) -> the
    GPU's (k, v) cache rows at `pos`; hist_rows(l) -> the (k, v) rows of positions 0..pos-1 (the
    oracle's, which the GPU was given).  Returns a dict: gemv_bad (non-bit-exact GEMV + residual
    values), quant_bad (quantisations outside the allowed flips), quant_flips (allowed flips), kv_bad
    (cache-row values differing from the replayed RoPE'd k / v), attn (worst rel error), swiglu (worst)."""
    import oracle as O

    L, hs = cfg.n_layers, cfg.dim // cfg.n_heads
    kv_mul = cfg.n_heads // cfg.n_kv_heads
    xres = gpu_xres(acts_g, L)
    out = {"gemv_bad": 0, "quant_bad": 0, "quant_flips": 0, "kv_bad": 0, "attn": 0.0, "swiglu": 0.0}
    # quantisation of each op's own input
    out["quant_detail"] = []
    for k, (gi, gq, gs) in enumerate(acts_g):
        if _is_norm_op(k, L):
            # The GPU's rmsnorm sums the squares in another order, so its scale factor r differs from the
            # restatement's by a few ulps, and so does every group scale (scale = max|w x r| / 127).  r
            # cancels in the quantiser's x * (1/scale): the int8 values may differ only where the
            # restatement's value lies within RMS_ULP_SLACK ulps of a rounding boundary, and every group's
            # scale ratio must be the same factor.
            xn = port.rmsnorm(np.ascontiguousarray(gi, np.float32), norm_w[k])
            q, s = port.quant_f32(xn)
            vp = pre_round(xn, s)
            for i in np.nonzero(q != gq)[0]:
                b = 0.5 * (int(q[i]) + int(gq[i]))
                ulp = float(np.spacing(np.float32(max(abs(vp[i]), 1.0))))
                if abs(int(q[i]) - int(gq[i])) == 1 and abs(float(vp[i]) - b) <= RMS_ULP_SLACK * ulp:
                    out["quant_flips"] += 1
                else:
                    out["quant_bad"] += 1
                    out["quant_detail"].append((k, int(i), int(q[i]), int(gq[i]), float(vp[i]), ulp))
            live = s != 0
            ratio = gs[live].astype(np.float64) / s[live].astype(np.float64)
            rho = float(np.median(ratio)) if ratio.size else 1.0
            nbad = int(np.count_nonzero(np.abs(ratio - rho) > 8 * 2.0 ** -23)) + int(abs(rho - 1.0) > 1e-5)
            out["quant_bad"] += nbad
            if nbad:
                out["quant_detail"].append((k, "scale ratio", rho, float(np.max(np.abs(ratio - rho)))))
        else:
            q, s = port.quant_f32(np.ascontiguousarray(gi, np.float32))
            out["quant_bad"] += int(np.count_nonzero(q != gq)) + int(np.count_nonzero(s.view(np.uint32) != gs.view(np.uint32)))
    cs = port.rope_coeffs(pos, hs)
    kv_dim = cfg.n_kv_heads * hs
    for l in range(L):
        # q|k|v from the GPU's activation (bit-exact GEMV), RoPE, the cache row the step wrote
        a = acts_g[4 * l]
        q = _rope(_mm(port, a, w[(O.PW_WQ, l)]), cs, cfg.n_heads, hs)
        kk = _rope(_mm(port, a, w[(O.PW_WK, l)]), cs, cfg.n_kv_heads, hs)
        vv = _mm(port, a, w[(O.PW_WV, l)])
        kg, vg = gpu_rows(l)
        kr = kk.astype(np.float32)
        if not kv_f32:  # bf16 truncation
            kt = (kr.view(np.uint32) >> 16).astype(np.uint16)
            vt = (vv.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
            out["kv_bad"] += int(np.count_nonzero(kt != kg.reshape(-1))) + int(np.count_nonzero(vt != vg.reshape(-1)))
        else:
            out["kv_bad"] += int(np.count_nonzero(kr.view(np.uint32) != kg.reshape(-1).view(np.uint32)))
            out["kv_bad"] += int(np.count_nonzero(vv.astype(np.float32).view(np.uint32) != vg.reshape(-1).view(np.uint32)))
        hk, hv = hist_rows(l)
        K = np.concatenate([_as_f64(hk).reshape(-1, kv_dim), _as_f64(kg).reshape(1, kv_dim)])
        V = np.concatenate([_as_f64(hv).reshape(-1, kv_dim), _as_f64(vg).reshape(1, kv_dim)])
        att = np.empty(cfg.dim)
        for h in range(cfg.n_heads):
            kh = (h // kv_mul) * hs
            sc = K[:, kh:kh + hs] @ q[h * hs:(h + 1) * hs].astype(np.float64) / np.sqrt(np.float64(hs))
            p = np.exp(sc - sc.max())
            att[h * hs:(h + 1) * hs] = (p / p.sum()) @ V[:, kh:kh + hs]
        out["attn"] = max(out["attn"], rel(acts_g[4 * l + 1][0], att))
        # wo + residual (bit-exact)
        x1 = (xres[2 * l] + _mm(port, acts_g[4 * l + 1], w[(O.PW_WO, l)])).astype(np.float32)
        out["gemv_bad"] += int(np.count_nonzero(x1.view(np.uint32) != xres[2 * l + 1].view(np.uint32)))
        # w1 / w3 from the GPU's activation (bit-exact GEMVs), SwiGLU in float64
        h1 = _mm(port, acts_g[4 * l + 2], w[(O.PW_W1, l)]).astype(np.float64)
        h3 = _mm(port, acts_g[4 * l + 2], w[(O.PW_W3, l)]).astype(np.float64)
        out["swiglu"] = max(out["swiglu"], rel(acts_g[4 * l + 3][0], h1 / (1.0 + np.exp(-h1)) * h3))
        # w2 + residual (bit-exact)
        x2 = (xres[2 * l + 1] + _mm(port, acts_g[4 * l + 3], w[(O.PW_W2, l)])).astype(np.float32)
        out["gemv_bad"] += int(np.count_nonzero(x2.view(np.uint32) != xres[2 * l + 2].view(np.uint32)))
    lg = _mm(port, acts_g[4 * L], w[(O.PW_WCLS, -1)])
    out["gemv_bad"] += int(np.count_nonzero(lg.view(np.uint32) != np.asarray(logits_g, np.float32).view(np.uint32)))
    return out


def synced_run(gpu, orc, seq, npos: int, port, w, norm_w, cfg):
    """Teacher-forced over `seq`, positions 0..npos-1, the GPU given the oracle's KV history before every
    step.  Returns per-position records (see the module docstring)."""
    L = cfg.n_layers
    names = op_names(L)
    recs = []
    hist = {l: [] for l in range(L)}
    for pos in range(npos):
        tok = int(seq[pos])
        if pos > 0:  # the oracle's rows of the previous position (earlier ones were written before)
            for l in range(L):
                k, v = orc.kv_rows(l, pos - 1, 1)
                gpu.kv_write(l, pos - 1, k, v)
                hist[l].append((k, v))
        lo, xo, ao = orc.forward_dump(tok, pos)
        lg = gpu.forward(tok, pos)
        ag = gpu.dump_read()
        xg = gpu_xres(ag, L)
        flips = cross_flips(ao, ag, norm_w, port, L)
        first = min((f["k"] for f in flips), default=len(names))
        cps = []
        for l in range(L):
            cps += [(f"L{l}.x", 4 * l, xo[2 * l], xg[2 * l]),
                    (f"L{l}.attn_out", 4 * l + 1, ao[4 * l + 1][0], ag[4 * l + 1][0]),
                    (f"L{l}.x_attn", 4 * l + 2, xo[2 * l + 1], xg[2 * l + 1]),
                    (f"L{l}.swiglu", 4 * l + 3, ao[4 * l + 3][0], ag[4 * l + 3][0])]
        # x_final is the classifier's input; the logits are its output, downstream of its activation
        cps += [("x_final", 4 * L, xo[2 * L], xg[2 * L]), ("logits", 4 * L + 1, lo, lg)]
        errs = [(name, rel(g, o)) for name, _, o, g in cps]
        # the input of op k is computed before op k's activation is quantised: clean when k <= first
        clean = [(name, rel(g, o)) for name, k, o, g in cps if k <= first]

        def hist_rows(l, _h=hist):
            if not _h[l]:
                return np.zeros((0, cfg.n_kv_heads * (cfg.dim // cfg.n_heads))), \
                    np.zeros((0, cfg.n_kv_heads * (cfg.dim // cfg.n_heads)))
            return np.concatenate([k for k, _ in _h[l]]), np.concatenate([v for _, v in _h[l]])

        ops = replay_ops(port, w, cfg, ag, lg, pos, lambda l: gpu.kv_read(l, pos, 1), hist_rows, norm_w,
                         getattr(gpu, "kv_f32", False))
        o = np.sort(lo)[-2:]
        recs.append({"pos": pos, "errs": errs, "clean": clean, "first_op": first,
                     "first_flips": [f for f in flips if f["k"] == first], "n_flips": len(flips), "ops": ops,
                     "top2_gap": float((o[1] - o[0]) / abs(o[1])), "logits_rel": rel(lg, lo),
                     "argmax": (int(np.argmax(lo)), int(np.argmax(lg)))})
    return recs


def check(recs, label):
    """The assertions over a synchronised run; returns a one-line summary."""
    for r in recs:
        op = r["ops"]
        assert op["gemv_bad"] == 0, (label, r["pos"], "GEMV replay not bit-exact", op)
        assert op["quant_bad"] == 0, (label, r["pos"], "quantisation outside boundary flips", op)
        assert op["kv_bad"] == 0, (label, r["pos"], "cache row differs from the replayed k / v", op)
        assert op["attn"] < OP_TOL and op["swiglu"] < OP_TOL, (label, r["pos"], op)
        bad = [f for f in r["first_flips"] if not f["explained"]]
        assert not bad, (label, r["pos"], "first flip not at a rounding boundary", bad[:4])
        worst = max(e for _, e in r["clean"])
        assert worst < REL_TOL, (label, r["pos"], [c for c in r["clean"] if c[1] >= REL_TOL])
    return summary(recs, label)


def summary(recs, label="") -> str:
    steps_with = sum(1 for r in recs if r["n_flips"])
    first = next((r["pos"] for r in recs if r["n_flips"]), None)
    worst_clean = max((e for r in recs for _, e in r["clean"]), default=0.0)
    worst_attn = max(r["ops"]["attn"] for r in recs)
    worst_sw = max(r["ops"]["swiglu"] for r in recs)
    qf = sum(r["ops"]["quant_flips"] for r in recs)
    return (f"{label}: {len(recs)} positions; {steps_with} steps with an int8 difference from the oracle (first "
            f"at position {first}); worst checkpoint error before a step's first difference {worst_clean:.2e}; "
            f"op replays: GEMVs bit-exact, {qf} rmsnorm-quantisation boundary flips, attention {worst_attn:.1e}, "
            f"SwiGLU {worst_sw:.1e}")


def synced_run_tp(gpu, orc, seq, npos: int, port, norm_w, cfg, rank: int, world: int):
    """synced_run for one tensor-parallel rank (every rank runs it in lockstep: each step exchanges
    partial sums).  The rank's checkpoints are compared with the oracle's -- the residual stream in full,
    the attention / SwiGLU outputs and the wo / w2 activations on this rank's slices (slices start at
    multiples of 32, so their Q8_0 groups are the oracle's) and this rank's classifier rows.  No op
    replays (the single-GPU runs make those): the split changes only the order in which wo's and w2's
    partial sums over the ranks are added."""
    from diolkos_b200 import tp

    L = cfg.n_layers
    sh = tp.shard(cfg, rank, world)
    names = op_names(L)
    recs = []
    for pos in range(npos):
        tok = int(seq[pos])
        if pos > 0:
            for l in range(L):
                k, v = orc.kv_rows(l, pos - 1, 1)
                gpu.kv_write(l, pos - 1, k, v)
        lo, xo, ao = orc.forward_dump(tok, pos)
        lg = gpu.forward(tok, pos)
        ag = gpu.dump_read()
        # the oracle's activations cut to this rank's slices where the GPU op holds a slice
        ao_s = []
        for k, (ai, aq, asc) in enumerate(ao):
            if k < 4 * L and k % 4 in (1, 3):
                c0, c1 = sh.q_rows if k % 4 == 1 else sh.hidden_rows
                ao_s.append((ai[c0:c1], aq[c0:c1], asc[c0 // 32:c1 // 32]))
            else:
                ao_s.append((ai, aq, asc))
        flips = cross_flips(ao_s, ag, norm_w, port, L)
        first = min((f["k"] for f in flips), default=len(names))
        xg = gpu_xres(ag, L)
        v0, v1 = sh.vocab_rows
        cps = []
        for l in range(L):
            cps += [(f"L{l}.x", 4 * l, xo[2 * l], xg[2 * l]),
                    (f"L{l}.attn_out", 4 * l + 1, ao_s[4 * l + 1][0], ag[4 * l + 1][0]),
                    (f"L{l}.x_attn", 4 * l + 2, xo[2 * l + 1], xg[2 * l + 1]),
                    (f"L{l}.swiglu", 4 * l + 3, ao_s[4 * l + 3][0], ag[4 * l + 3][0])]
        cps += [("x_final", 4 * L, xo[2 * L], xg[2 * L]), ("logits", 4 * L + 1, lo[v0:v1], lg[v0:v1])]
        clean = [(name, rel(g, o)) for name, k, o, g in cps if k <= first]
        recs.append({"pos": pos, "clean": clean, "first_op": first, "n_flips": len(flips),
                     "first_flips": [f for f in flips if f["k"] == first], "logits_rel": rel(lg[v0:v1], lo[v0:v1])})
    return recs


def check_tp(recs, label):
    for r in recs:
        bad = [f for f in r["first_flips"] if not f["explained"]]
        assert not bad, (label, r["pos"], "first flip not at a rounding boundary", bad[:4])
        worst = max(e for _, e in r["clean"])
        assert worst < REL_TOL, (label, r["pos"], [c for c in r["clean"] if c[1] >= REL_TOL])
    steps_with = sum(1 for r in recs if r["n_flips"])
    worst_clean = max((e for r in recs for _, e in r["clean"]), default=0.0)
    return (f"{label}: {len(recs)} positions; {steps_with} steps with an int8 difference from the oracle; worst "
            f"checkpoint error before a step's first difference {worst_clean:.2e}")
