"""Generates tests/golden/c4_greedy.npz: the CPU oracle's greedy token stream
for the benchmark's dense decoder (configuration 4: 35 layers, hidden 1536,
8 query heads / 1 KV head of 256, FFN 6144, vocab 262144, all Q8_0; seeded
random-init weights, seed 3), from <bos> + 128 uniform random prompt ids,
256 generated tokens.  Also stores, per generated token, the gap between the
two largest logits (how close the argmax was to a tie), and how far the
logits of the reference's other dot-product mode (scalarDot everywhere, the
llama.VectorBitSize=0 switch) are from these over the first 8 positions: the
size of a pure summation-order difference on this model.

    python tests/golden/make_decode_golden.py

Uses only the oracle (oracle/g4_oracle.c, the restatement of Llama.forward)
and the build's seeded generator (gemma4.kt_b200/synth.py).
"""
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from gemma4_kt_b200 import synth  # noqa: E402
from gemma4_kt_b200.model import TensorSource  # noqa: E402
from oracle import oracle  # noqa: E402

SEED, N_PROMPT, N_GEN = 3, 128, 256


def main():
    t0 = time.time()
    m = synth.SynthDecoder(synth.C4_DENSE, seed=SEED)
    prompt = m.prompt(N_PROMPT)
    print(f"model generated in {time.time() - t0:.1f} s", flush=True)
    orc = oracle.ModelOracle(TensorSource.from_synth(m))
    t0 = time.time()
    toks, logits = orc.greedy(prompt, N_GEN, collect_logits=True)
    gen_logits = logits[N_PROMPT:]
    gaps = np.array([float(np.diff(np.sort(lg)[-2:])[0]) for lg in gen_logits], np.float32)
    print(f"oracle decode of {N_PROMPT + 1 + N_GEN} positions in {time.time() - t0:.1f} s; "
          f"smallest top-2 gap {gaps.min():.3e}", flush=True)
    orc.close()
    oracle.set_vector_api(False)
    scalar = oracle.ModelOracle(TensorSource.from_synth(m))
    toks_in = [2] + [int(t) for t in prompt]
    rel = []
    for p in range(8):
        lg = scalar.step(toks_in[p], p)
        rel.append(float(np.linalg.norm(lg - logits[p]) / np.linalg.norm(logits[p])))
    oracle.set_vector_api(True)
    print(f"scalarDot vs Vector-API logits, positions 0-7: max rel L2 {max(rel):.3e}", flush=True)
    np.savez_compressed(Path(__file__).with_name("c4_greedy.npz"), seed=SEED, prompt=prompt, generated=toks,
                        top2_gap=gaps, scalar_vs_vector_rel=np.array(rel, np.float32))


if __name__ == "__main__":
    main()
