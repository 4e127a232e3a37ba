"""The conversion partition (``convert.prepare_ar``; conversion.cpp:203-300, :440-475) on a
synthetic upstream checkpoint: AR and NAR tensors together in two shards with an index.
The AR file must hold the AR tensors byte for byte in the loader's order, the NAR file the
rest, the manifest one record per precision and a digest per file; the loader accepts the
directory (on CPU it gets as far as the device), and on a GPU decodes the same logits as
the directory the tensors came from."""
import dataclasses
import json
import os

import numpy as np
import pytest

from tests.conftest import ROOT, _load


@pytest.fixture(scope="module")
def conv():
    return _load("yue2_mlx_b200_convert", os.path.join(ROOT, "yue2-mlx_b200", "convert.py"))


@pytest.fixture(scope="module")
def small_dims(synth):
    return dataclasses.replace(synth.TINY, ffn=512, vocab=512, context=256)


def _config(synth, dims):
    c = dict(synth.config_json(dims))
    c.update(model_type="yue2", architectures=["YuE2ForCausalLM"], latent_type="vae", latent_dim=64,
             max_latent_frames=dims.context, timestep_shift=1.0, dtype="bfloat16")
    return c


def _write_st(path, tensors):
    header, off, blobs = {}, 0, []
    for name, arr in tensors:
        b = np.ascontiguousarray(arr).view(np.uint8).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    raw = json.dumps(header).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(np.uint64(len(raw)).tobytes() + raw + b"".join(blobs))


@pytest.fixture(scope="module")
def upstream(synth, small_dims, tmp_path_factory):
    """Two shards: NAR tensors and half the AR tensors in one, the rest in the other, in an
    order unlike the loader's."""
    src = tmp_path_factory.mktemp("conv_src")
    ref = str(tmp_path_factory.mktemp("conv_ref"))
    synth.write_converted(ref, small_dims, seed=11, norm_std=0.1, workers=2)
    ar = synth.read_safetensors(os.path.join(ref, "ar-bf16.safetensors"))
    rng = np.random.default_rng(0)
    nar = [("llm2vae.weight", rng.integers(0, 65535, (64, small_dims.hidden), dtype=np.uint16)),
           ("model.layers.0.nar_self_attn.q_proj.weight", rng.integers(0, 65535, (8, 8), dtype=np.uint16)),
           ("latent_pos_embed.pe", rng.integers(0, 65535, (4, small_dims.hidden), dtype=np.uint16))]
    names = list(ar)[::-1]
    half = len(names) // 2
    _write_st(str(src / "model-00001-of-00002.safetensors"), nar[:2] + [(n, ar[n]) for n in names[:half]])
    _write_st(str(src / "model-00002-of-00002.safetensors"), [(n, ar[n]) for n in names[half:]] + nar[2:])
    wm = {n: "model-00001-of-00002.safetensors" for n, _ in nar[:2]}
    wm.update({n: "model-00001-of-00002.safetensors" for n in names[:half]})
    wm.update({n: "model-00002-of-00002.safetensors" for n in names[half:]})
    wm[nar[2][0]] = "model-00002-of-00002.safetensors"
    json.dump({"weight_map": wm}, open(src / "model.safetensors.index.json", "w"))
    json.dump(_config(synth, small_dims), open(src / "config.json", "w"))
    return str(src), ref, ar, dict(nar)


def test_partition_and_manifest(conv, synth, upstream, tmp_path):
    src, ref, ar, nar = upstream
    out = conv.prepare_ar(src, str(tmp_path / "out"), precisions=("bf16", "8bit"), any_dims=True)
    # The AR file equals the synthetic writer's byte for byte (same tensors, same order).
    assert open(os.path.join(out, "ar-bf16.safetensors"), "rb").read()[8:].split(b"}", 1)[1].lstrip(b" ") == \
        open(os.path.join(ref, "ar-bf16.safetensors"), "rb").read()[8:].split(b"}", 1)[1].lstrip(b" ")
    got = synth.read_safetensors(os.path.join(out, "ar-bf16.safetensors"))
    assert list(got) == list(synth.read_safetensors(os.path.join(ref, "ar-bf16.safetensors")))
    for n, v in ar.items():
        np.testing.assert_array_equal(got[n], v)
    gn = synth.read_safetensors(os.path.join(out, "nar-bf16.safetensors"))
    assert set(gn) == set(nar)
    for n, v in nar.items():
        np.testing.assert_array_equal(gn[n], v)
    man = json.load(open(os.path.join(out, "conversion.json")))
    assert man["schema"] == 1 and set(man["precisions"]) == {"bf16", "8bit"}
    assert man["precisions"]["bf16"]["ar"] == "ar-bf16.safetensors"
    assert man["precisions"]["8bit"]["bits"] == 8 and man["precisions"]["8bit"]["group_size"] == 64
    for name, rec in man["files"].items():
        assert rec == conv.file_record(os.path.join(out, name))
    # The 8-bit file is the quantization of these same weights.
    q_ref = str(tmp_path / "q_ref")
    os.makedirs(q_ref)
    os.link(os.path.join(ref, "ar-bf16.safetensors"), os.path.join(q_ref, "ar-bf16.safetensors"))
    synth.write_quantized(q_ref, synth.Dims(**{**dataclasses.asdict(synth.TINY), "ffn": 512, "vocab": 512,
                                               "context": 256}))
    assert open(os.path.join(q_ref, "ar-8bit.safetensors"), "rb").read() == \
        open(os.path.join(out, "ar-8bit.safetensors"), "rb").read()


def test_loader_accepts_the_prepared_directory(conv, upstream, tmp_path):
    yar = _load("yue2_mlx_b200", os.path.join(ROOT, "yue2-mlx_b200", "__init__.py"),
                os.path.join(ROOT, "yue2-mlx_b200"))
    src, _, _, _ = upstream
    out = conv.prepare_ar(src, str(tmp_path / "out"), precisions=("bf16", "8bit"), any_dims=True)
    from tests.conftest import has_gpu
    if has_gpu():
        pytest.skip("covered by the GPU test below")
    for precision in ("bf16", "8bit"):
        with pytest.raises(yar.YarError) as e:  # every check passed; no device here
            yar.ARModel(out, any_dims=True, precision=precision)
        assert e.value.kind == "RuntimeError" and "CUDA" in e.value.message, e.value.message


@pytest.mark.parametrize("edit,needle", [
    (lambda c: c.update(hidden_size=4096), "Pinned generator config mismatch: hidden_size"),
    (lambda c: c.update(tie_word_embeddings=True), "tie_word_embeddings"),
    (lambda c: c.update(dtype="float32"), "bfloat16"),
])
def test_config_checks(conv, synth, edit, needle):
    c = _config(synth, synth.PINNED)
    conv.validate_config(c)  # the pinned config passes as written
    edit(c)
    with pytest.raises(ValueError, match=needle):
        conv.validate_config(c)


def test_missing_tensor_is_an_error(conv, synth, upstream, tmp_path):
    src, _, ar, _ = upstream
    idx = json.load(open(os.path.join(src, "model.safetensors.index.json")))
    cut = str(tmp_path / "cut")
    os.makedirs(cut)
    keep = [n for n in ar if n != "model.layers.1.mlp.up_proj.weight"]
    _write_st(os.path.join(cut, "model.safetensors"), [(n, ar[n]) for n in keep])
    json.dump(json.load(open(os.path.join(src, "config.json"))), open(os.path.join(cut, "config.json"), "w"))
    assert "weight_map" in idx
    with pytest.raises(ValueError, match="Missing partition tensors"):
        conv.prepare_ar(cut, str(tmp_path / "out"), any_dims=True)


@pytest.mark.gpu
def test_prepared_directory_decodes_like_its_source(conv, upstream, tmp_path):
    yar = _load("yue2_mlx_b200", os.path.join(ROOT, "yue2-mlx_b200", "__init__.py"),
                os.path.join(ROOT, "yue2-mlx_b200"))
    src, ref, _, _ = upstream
    out = conv.prepare_ar(src, str(tmp_path / "out"), any_dims=True)
    prompt = list(range(3, 60))
    logits = []
    for d in (out, ref):
        m = yar.ARModel(d, any_dims=True)
        s = m.session(max_rows=1, max_ctx=128)
        s.reset(0, 128)
        s.prefill(0, prompt, phase=None)
        s.step([0], [7], phase=None)
        logits.append(s.logits(0, None))
        s.close()
        m.close()
    np.testing.assert_array_equal(logits[0], logits[1])
