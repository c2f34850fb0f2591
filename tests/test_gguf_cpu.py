"""The synthetic GGUF writer and the reader the model loader uses
(GGUF.kt:89-212, ModelLoader.kt:39-261): a generated decoder written to a
file and read back gives the same metadata, tensor infos and block bytes,
the loader's configuration, and the same oracle logits as the in-memory
model.  Malformed headers are refused the way the reference refuses them."""
import struct

import numpy as np
import pytest

from oracle import oracle


def _tiny(**kw):
    from gemma4_kt_b200 import synth

    base = dict(name="tiny", n_layers=3, dim=256, n_heads=2, n_kv_heads=1, head_size=128, ff=512, vocab=600,
                ctx_len=32, sliding_window=8, swa_period=2, shared_kv_layers=1, no_v_layers=(1,))
    base.update(kw)
    return synth.DecoderSpec(**base)


@pytest.fixture(scope="module")
def written(g4, tmp_path_factory):
    from gemma4_kt_b200 import synth

    m = synth.SynthDecoder(_tiny(), seed=5)
    path = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    m.write(path)
    return m, path


def test_round_trip_metadata_and_tensors(g4, written):
    from gemma4_kt_b200 import gguf

    m, path = written
    f = gguf.GGUFFile(path)
    assert f.version == 3 and f.alignment == 32
    assert f.data_offset % 32 == 0
    assert set(f.metadata) == set(m.metadata)
    for k, v in m.metadata.items():
        want = v.value if isinstance(v, gguf.Typed) else v
        got = f.metadata[k]
        if isinstance(want, (list, tuple, np.ndarray)):
            got, want = list(got), list(want)
            if want and isinstance(want[0], (float, np.floating)):
                np.testing.assert_array_equal(np.asarray(got, np.float32), np.asarray(want, np.float32))
            else:
                assert got == want, k
        elif isinstance(want, float):
            assert np.float32(got) == np.float32(want), k
        else:
            assert got == want, k
    assert list(f.tensors) == [t[0] for t in m.tensors]  # file order kept
    for name, dims, gt, raw in m.tensors:
        ti = f.tensors[name]
        assert ti.dims == tuple(dims) and ti.ggml_type == gt and ti.offset % 32 == 0
        assert np.array_equal(np.asarray(f.tensor_bytes(name)), np.asarray(raw).view(np.uint8).reshape(-1)), name


def test_loader_config_from_file(g4, written):
    m, path = written
    from gemma4_kt_b200 import gguf

    a = g4.TensorSource.from_gguf(gguf.GGUFFile(path)).config()
    b = g4.TensorSource.from_synth(m).config()
    assert a == b
    s = m.spec
    assert (a.dim, a.n_layers, a.n_heads, a.vocab, a.ctx_len) == (s.dim, s.n_layers, s.n_heads, s.vocab, s.ctx_len)
    assert a.is_swa == [s.is_swa(l) for l in range(s.n_layers)]
    assert a.n_layer_kv_from_start == s.n_layers - s.shared_kv_layers
    # the tokenizer arrays carry the special tokens the chat format looks up
    toks = gguf.GGUFFile(path).metadata["tokenizer.ggml.tokens"]
    for t in ("<bos>", "<eos>", "<|turn>", "<turn|>", "<0x00>"):
        assert t in toks


def test_oracle_same_logits_from_file(g4, written):
    """The oracle's forward over the file's bytes equals the in-memory one bit for bit."""
    from gemma4_kt_b200 import gguf

    m, path = written
    a = oracle.ModelOracle(g4.TensorSource.from_gguf(gguf.GGUFFile(path)))
    b = oracle.ModelOracle(g4.TensorSource.from_synth(m))
    tok = 2
    for pos in range(4):
        la, lb = a.step(tok, pos), b.step(tok, pos)
        assert np.array_equal(la, lb)
        tok = int(np.argmax(la))
    a.close()
    b.close()


def _header(magic=0x46554747, version=3):
    return struct.pack("<IIQQ", magic, version, 0, 0)


@pytest.mark.parametrize("magic,version,err", [(0x12345678, 3, "magic"), (0x46554747, 1, "version")])
def test_reader_rejects_bad_header(g4, tmp_path, magic, version, err):
    from gemma4_kt_b200 import gguf

    p = tmp_path / "bad.gguf"
    p.write_bytes(_header(magic, version) + b"\0" * 32)
    with pytest.raises(ValueError, match=err):
        gguf.GGUFFile(p)


def test_reader_rejects_misaligned_tensor(g4, tmp_path):
    from gemma4_kt_b200 import gguf

    name = b"t"
    body = struct.pack("<IIQQ", 0x46554747, 3, 1, 0)
    body += struct.pack("<Q", len(name)) + name + struct.pack("<I", 1) + struct.pack("<Q", 8)
    body += struct.pack("<IQ", 0, 4)  # F32, offset 4: not a multiple of 32
    p = tmp_path / "mis.gguf"
    p.write_bytes(body + b"\0" * 128)
    with pytest.raises(ValueError, match="aligned"):
        gguf.GGUFFile(p)


def test_writer_refuses_wrong_byte_count(g4, tmp_path):
    from gemma4_kt_b200 import gguf

    with pytest.raises(ValueError):
        gguf.write_gguf(tmp_path / "x.gguf", {}, [("w", (32,), g4.GGMLType.Q8_0, np.zeros(30, np.uint8))])
