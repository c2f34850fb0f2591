"""GPU parity of the whole-model decoder (g4_model / g4_state / g4_decode_*,
Llama.kt:105-477) against the CPU oracle's restatement of Llama.forward.

Small synthetic models cover the features of the forward pass: sliding-window
and full attention (RoPE tables of both kinds), GQA at several query heads per
KV head, shared-KV layers, a layer without attn_v (V = K), layer output
scales, logit softcapping, every fast weight format, and MoE layers (shared
MLP + experts + merge).  Every step's logits must be within 1e-3 relative L2
of the oracle's and the greedy token streams identical.  The benchmark's
dense decoder (configuration 4: 35 layers, Q8_0, vocab 262144, seed 3) is
compared with the oracle's greedy stream (committed fixture,
tests/golden/make_decode_golden.py).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
GOLDEN = Path(__file__).resolve().parent / "golden" / "c4_greedy.npz"


def _spec(**kw):
    from gemma4_kt_b200 import synth

    base = dict(name="tiny", n_layers=4, dim=512, n_heads=4, n_kv_heads=2, head_size=128, ff=1024, vocab=2048,
                ctx_len=160, sliding_window=16, swa_period=3)
    base.update(kw)
    return synth.DecoderSpec(**base)


SPECS = {
    "q8-swa-shared-noV": _spec(shared_kv_layers=1, no_v_layers=(1,)),
    "q8-gqa8": _spec(n_heads=8, n_kv_heads=1, head_size=64, swa_period=0),
    "q4k": _spec(wtype=12, emb_type=12, n_kv_heads=4, head_size=128),
    "q6k-mha": _spec(wtype=14, emb_type=14, n_heads=4, n_kv_heads=4, head_size=64, softcap=0.0),
    "bf16": _spec(wtype=30, emb_type=30, n_layers=2, layer_scale=False),
    "moe": _spec(n_layers=3, ff=512, n_expert=16, n_expert_used=4, expert_ff=256, shared_kv_layers=0),
}

# Seeds of the MoE model: an expert choice is only reproducible where the
# k-th and (k+1)-th router probabilities differ by more than fp32 rounding.
# With 16 experts and ~250 routings per run, many seeds hold a gap near
# 1e-7 somewhere (a tie: the oracle's own Vector-API and scalarDot modes
# differ by that much), so these seeds keep every gap of the run above
# MIN_MARGIN, which the tests check on the oracle.
SEEDS = {"moe": 39}
MIN_MARGIN = 2e-6


def _check_margin(name):
    if SPECS[name].n_expert:
        assert oracle.topk_margin() >= MIN_MARGIN, (name, "ill-conditioned fixture", oracle.topk_margin())


def _models(g4, ctx, spec, seed):
    from gemma4_kt_b200 import synth

    m = synth.SynthDecoder(spec, seed=seed)
    src = g4.TensorSource.from_synth(m)
    return m, src, g4.DecoderModel(ctx, src), oracle.ModelOracle(src)


@pytest.mark.parametrize("name", list(SPECS))
def test_decode_steps_vs_oracle(g4, ctx, name):
    """Prompt and greedy steps one at a time through g4_decode_step: logits of
    every step vs the oracle, and the argmax fed back identically."""
    m, src, model, orc = _models(g4, ctx, SPECS[name], seed=SEEDS.get(name, 11))
    st = model.new_state()
    prompt = m.prompt(40)
    token, pos, errs = 2, 0, []
    oracle.reset_topk_margin()
    for i in range(80):
        lg, nt = st.step(token, pos)
        ref = orc.step(token, pos)
        errs.append(rel_l2(lg, ref))
        assert errs[-1] < TOL, (name, pos, errs[-1])
        assert nt == int(np.argmax(lg))
        if i < len(prompt):
            token = int(prompt[i])
        else:
            assert nt == int(np.argmax(ref)), (name, pos)
            token = nt
        pos += 1
    _check_margin(name)
    print(f"\n{name}: per-step logits rel L2 max {max(errs):.2e} mean {np.mean(errs):.2e}")
    st.free()
    model.free()


@pytest.mark.parametrize("name", ["q8-swa-shared-noV", "moe"])
def test_greedy_stream_gpu_resident(g4, ctx, name):
    """g4_decode_greedy (argmax fed back on the device, no host round trip)
    gives the oracle's token stream over 64 generated tokens, and a second
    run on a fresh state repeats it exactly."""
    m, src, model, orc = _models(g4, ctx, SPECS[name], seed=SEEDS.get(name, 12))
    prompt = m.prompt(24)
    oracle.reset_topk_margin()
    ref = orc.greedy(prompt, 64)
    _check_margin(name)
    st = model.new_state()
    got = st.generate(np.concatenate([[2], prompt]).astype(np.int32), 64)
    assert np.array_equal(got, ref), (name, got, ref)
    st2 = model.new_state()
    again = st2.generate(np.concatenate([[2], prompt]).astype(np.int32), 64)
    np.testing.assert_array_equal(again, got)
    st.free()
    st2.free()
    model.free()


def test_decoder_rejects_bad_input(g4, ctx):
    m, src, model, _ = _models(g4, ctx, SPECS["bf16"], seed=13)
    st = model.new_state()
    with pytest.raises(g4.G4Error):
        st.step(model.cfg.vocab, 0)
    with pytest.raises(g4.G4Error):
        st.step(0, model.cfg.ctx_len)
    with pytest.raises(g4.G4Error):
        st.generate(np.array([2, 5], np.int32), model.cfg.ctx_len)
    st.free()
    model.free()


def test_c4_dense_greedy_64_tokens(g4, ctx):
    """Configuration 4 at full size: 35 layers, hidden 1536, 8 query heads and
    1 KV head of 256, FFN 6144, vocab 262144, all Q8_0, seed 3; BOS + 128
    random prompt ids, then greedy decode.  The first 64 generated tokens equal
    the oracle's (fixture); the rest are reported."""
    from gemma4_kt_b200 import synth

    gold = np.load(GOLDEN)
    m = synth.SynthDecoder(synth.C4_DENSE, seed=int(gold["seed"]))
    prompt = m.prompt(128)
    np.testing.assert_array_equal(prompt, gold["prompt"])
    model = g4.DecoderModel(ctx, g4.TensorSource.from_synth(m))
    del m
    st = model.new_state()
    n = int(gold["generated"].size)
    got = st.generate(np.concatenate([[2], prompt]).astype(np.int32), n)
    ref = gold["generated"]
    first_diff = int(np.argmax(got != ref)) if np.any(got != ref) else n
    print(f"\nC4 greedy: first difference at generated token {first_diff} of {n}")
    assert first_diff >= 64, (first_diff, got[:first_diff + 1], ref[:first_diff + 1])
    st.free()
    model.free()


def test_decoder_from_gguf_file(g4, ctx, tmp_path):
    """GemmaModel.load's path: a synthetic decoder written as a GGUF file and
    loaded with DecoderModel.load (mmapped blocks uploaded as they lie)
    decodes the same greedy stream as the oracle."""
    from gemma4_kt_b200 import gguf, synth

    m = synth.SynthDecoder(SPECS["q4k"], seed=14)
    path = tmp_path / "q4k.gguf"
    m.write(path)
    prompt = m.prompt(12)
    del m
    model = g4.DecoderModel.load(ctx, path)
    orc = oracle.ModelOracle(g4.TensorSource.from_gguf(gguf.GGUFFile(path)))
    ref = orc.greedy(prompt, 24)
    st = model.new_state()
    got = st.generate(np.concatenate([[2], prompt]).astype(np.int32), 24)
    assert np.array_equal(got, ref), (got, ref)
    st.free()
    model.free()


C5_GOLDEN = Path(__file__).resolve().parent / "golden" / "c5_greedy.npz"


def _batched_stream(model, toks, n):
    """<bos> + prompt prefilled in 64-row chunks of one slot, then n - 1 single-row steps."""
    b = model.new_batch(64, toks.size + n)
    nt = None
    for p0 in range(0, toks.size, 64):
        p1 = min(p0 + 64, toks.size)
        _, nt = b.step(toks[p0:p1], np.arange(p0, p1, dtype=np.int32), want_logits=False,
                       slots=np.zeros(p1 - p0, np.int32))
    gen = [int(nt[-1])]
    for i in range(n - 1):
        _, nt = b.step([gen[-1]], [toks.size + i], want_logits=False)
        gen.append(int(nt[0]))
    b.free()
    return np.array(gen, np.int32)


def test_c5_moe_greedy_64_tokens(g4, ctx, monkeypatch):
    """Configuration 5 geometry at full size (MoE decoder, seed 4; the layer
    matrices shared by the 30 layers as in the benchmark), one sequence:
    <bos> + 512 random prompt ids, then greedy decode.  The single-sequence
    decoder (one CUDA graph per step, the MoE layers on the one-token decode
    kernels) must give the oracle's 64 tokens (fixture,
    tests/golden/make_c5_golden.py), and so must the batched decoder (the
    prompt prefilled in 64-row chunks of one slot) with the chunks' MoE
    layers on the fp32 CUDA-core expert kernels.  With the chunks' experts on
    the tensor-core path (fp16 weights, ~5e-4 per token) the stream is only
    reported: it leaves the oracle's after about 20 tokens on this fixture."""
    import dataclasses

    from gemma4_kt_b200 import synth

    gold = np.load(C5_GOLDEN)
    m = synth.SynthDecoder(dataclasses.replace(synth.C5_MOE, replicate_layers=True), seed=int(gold["seed"]))
    prompt = m.prompt(512)
    np.testing.assert_array_equal(prompt, gold["prompt"])
    model = g4.DecoderModel(ctx, g4.TensorSource.from_synth(m))
    del m
    ref = gold["generated"]
    n = ref.size
    toks = np.concatenate([[2], prompt]).astype(np.int32)
    st = model.new_state()
    got = st.generate(toks, n)
    st.free()

    def first_diff(a):
        return int(np.argmax(a != ref)) if np.any(a != ref) else n

    monkeypatch.setenv("G4_MOE_TC", "0")
    first_cc = first_diff(_batched_stream(model, toks, n))
    monkeypatch.setenv("G4_MOE_TC", "1")
    first_tc = first_diff(_batched_stream(model, toks, n))
    model.free()
    print(f"\nC5 greedy (smallest routing margin of the oracle run {float(gold['topk_margin']):.1e}): first "
          f"difference at generated token {first_diff(got)} of {n} (decoder); batched prefill + decode: "
          f"{first_cc} (CUDA-core experts), {first_tc} (tensor-core experts)")
    assert first_diff(got) == n, (got, ref)
    assert first_cc == n, first_cc
