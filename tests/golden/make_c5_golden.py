"""Generates tests/golden/c5_greedy.npz: the CPU oracle's greedy token stream
for one sequence of the benchmark's MoE decoder (configuration 5: 30 layers,
hidden 2816, 16 query / 8 KV heads of 256, 128 experts top-8 with ff 704 in
Q4_K, a shared 2112-wide Q8_0 FFN, vocab 262144; seed 4) from <bos> + 512
uniform random prompt ids, 64 generated tokens.  As in the benchmark, the
layer matrices are generated once and used by all 30 layers (norm weights
and scales are drawn per layer); generating 15 GB of distinct experts on the
host would take tens of minutes.  Also stores the smallest routing margin of
the run (oracle.topk_margin: the gap between the 8th and 9th router
probability) and the top-2 logit gap of each generated token.

    python tests/golden/make_c5_golden.py

Uses only the oracle (oracle/g4_oracle.c) and the build's seeded generator.
"""
import dataclasses
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

SEED, N_PROMPT, N_GEN = 4, 512, 64
SPEC = dataclasses.replace(synth.C5_MOE, replicate_layers=True)


def main():
    t0 = time.time()
    m = synth.SynthDecoder(SPEC, seed=SEED)
    prompt = m.prompt(N_PROMPT)
    print(f"model generated in {time.time() - t0:.1f} s", flush=True)
    orc = oracle.ModelOracle(TensorSource.from_synth(m), context_length=N_PROMPT + N_GEN + 1)
    t0 = time.time()
    oracle.reset_topk_margin()
    toks, logits = orc.greedy(prompt, N_GEN, collect_logits=True)
    margin = oracle.topk_margin()
    gaps = np.array([float(np.diff(np.sort(lg)[-2:])[0]) for lg in logits[N_PROMPT:]], np.float32)
    print(f"oracle decode of {N_PROMPT + N_GEN} positions in {time.time() - t0:.1f} s; smallest routing margin "
          f"{margin:.3e}; smallest top-2 gap {gaps.min():.3e}", flush=True)
    orc.close()
    np.savez_compressed(Path(__file__).with_name("c5_greedy.npz"), seed=SEED, prompt=prompt, generated=toks,
                        top2_gap=gaps, topk_margin=np.float64(margin))


if __name__ == "__main__":
    main()
