"""Generate tests/golden/llama7b_greedy.json: the reference's greedy stream of the decode benchmark's
workload (LLaMA-2-7B shape, seeded weights, 32-token seeded prompt, 256 greedy tokens).

The weights are the benchmark's own: generated on a GPU from bench.SEED (torch's CUDA generator) and
quantised by the library's quantiser, which is bit-exact with the reference loader's; they reach the
reference as its Q8_0 cache files.  The stream comes from the reference's own generate loop
(oracle/ref_driver.c: oref_generate over the unmodified sources, portable -march=x86-64-v3 build, whose
arithmetic does not depend on the host CPU), with the top-2 logits at every generated position.
bench.py compares its greedy tokens with this stream at every GPU count, free-running and teacher-forced;
the fixture also holds the teacher-forced agreement of the oracle's restatement with the stream, the
control for that count.

Run on a machine with a GPU and oracle/_ref built:
    python tests/golden/make_llama7b_stream.py [out.json]
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def main(out_path: str) -> None:
    import torch

    import bench
    from diolkos_b200 import synth
    from oracle import Ref

    cfg, P, G, _ = bench._models()["7b"]
    torch.cuda.set_device(0)
    ref = Ref("portable")
    cores = ref.threads(bench.physical_cores())
    tmp = tempfile.mkdtemp(prefix="dk_stream_")
    md = bench.write_reference_model(tmp, cfg, bench.SEED)
    m = ref.load(md, tmp)
    prompt = synth.seeded_prompt(bench.SEED, P, cfg.vocab_size)
    toks, secs, top2 = m.generate_timed(prompt, P - 1 + G)
    doc = {"seed": bench.SEED, "prompt": [int(t) for t in prompt], "tokens": [int(t) for t in toks],
           "top2": [[float(a), float(b)] for a, b in top2],
           "reference": "oracle/_ref portable build (unmodified reference, -Ofast -march=x86-64-v3), oref_generate",
           "model": "llama2-7b-shape, seeded N(0,0.02) weights generated on the GPU (bench.host_weights)",
           "cpu_seconds": round(secs, 2), "cpu_threads": cores}
    # The control for bench.py's teacher-forced check: the oracle's restatement (oracle/port.c, the
    # reference's arithmetic in the reference's order, bit-exact for the integer work, but glibc's scalar
    # expf / sqrtf where the -Ofast reference build calls libmvec's vector expf) fed the same stream.
    os.environ["OMP_NUM_THREADS"] = str(cores)
    pm = bench.port_model(cfg, bench.SEED)
    ctl = bench.forced_check(pm, prompt, doc["tokens"], doc["top2"], 1, "oracle/port.c restatement")
    doc["control_forced"] = {k: ctl[k] for k in ("agree", "of", "max_gap_at_disagreement")}
    doc["control_forced"]["what"] = ("oracle/port.c restatement (glibc scalar expf; otherwise the reference's "
                                     "arithmetic and order), teacher-forced with this stream, bf16 KV")
    doc["control_forced"]["disagreements"] = ctl["disagreements"]
    with open(out_path, "w") as f:
        json.dump(doc, f)
    import shutil

    shutil.rmtree(tmp, ignore_errors=True)
    print(f"wrote {out_path}: {len(toks)} tokens in {secs:.1f} s on {cores} threads")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "llama7b_greedy.json"))
