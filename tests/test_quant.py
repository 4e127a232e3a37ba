"""The `8bit` and `4bit` precisions without a GPU: the synthetic artifacts have the reference's layout
(conversion.py:596-620, :754-761), the oracle's dequantization follows the published
affine group-64 semantics, and the loader rejects bad 8-bit checkpoints with the
reference's messages (native/src/ar.cpp:137-160, :193-236) before touching the device."""
import dataclasses
import json
import os
import shutil

import numpy as np
import pytest

from oracle import ar_oracle as ora
from tests.conftest import load_package

pytestmark = pytest.mark.filterwarnings("ignore::DeprecationWarning")


@pytest.fixture(scope="module")
def yar():
    return load_package()


@pytest.fixture(scope="module")
def q8_dims(synth):
    # Every linear input width a multiple of 64 (the tiny config's FFN of 688 is not).
    return dataclasses.replace(synth.TINY, ffn=512, vocab=512, context=256)


@pytest.fixture(scope="module")
def q8_dir(tmp_path_factory, synth, q8_dims):
    d = str(tmp_path_factory.mktemp("q8small"))
    synth.write_converted(d, q8_dims, seed=5, norm_std=0.1, workers=2, precisions=("bf16", "8bit", "4bit"))
    return d


def test_artifact_layout(synth, q8_dir, q8_dims):
    man = json.load(open(os.path.join(q8_dir, "conversion.json")))
    assert man["precisions"]["8bit"] == {"ar": "ar-8bit.safetensors", "bits": 8, "group_size": 64,
                                         "mode": "affine", "linear_only": True, "embedding_dtype": "bfloat16"}
    q = synth.read_safetensors(os.path.join(q8_dir, "ar-8bit.safetensors"))
    b = synth.read_safetensors(os.path.join(q8_dir, "ar-bf16.safetensors"))
    linear = set(synth.linear_names(q8_dims))
    assert "model.embed_tokens.weight" not in linear and "lm_head.weight" in linear
    for name, bits in b.items():
        if name in linear:
            out, inp = bits.shape
            p = name[: -len("weight")]
            assert q[name].dtype == np.uint32 and q[name].shape == (out, inp // 4)
            assert q[p + "scales"].shape == (out, inp // 64) and q[p + "biases"].shape == (out, inp // 64)
        else:
            np.testing.assert_array_equal(q[name], bits)
    assert len(q) == len(b) + 2 * len(linear)


def test_quantizer_reconstructs_within_one_step(synth):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((48, 256)) * 0.02).astype(np.float32)
    w[3, :64] = 0.5  # a constant group: scale clamps at its floor, q is 0
    q, s_bits, b_bits = synth.quantize_affine8(w)
    s, b = synth.bf16_bits_to_f32(s_bits), synth.bf16_bits_to_f32(b_bits)
    deq = q.astype(np.float32).reshape(48, 4, 64) * s[:, :, None] + b[:, :, None]
    err = np.abs(deq - w.reshape(48, 4, 64))
    # Half a step from rounding q, plus the BF16 rounding of scale and bias.
    assert np.all(err <= s[:, :, None] * 0.5 + np.abs(b)[:, :, None] * 2.0 ** -8 + 255 * s[:, :, None] * 2.0 ** -8)
    assert q[3, :64].max() == 0 and abs(deq[3, 0, 0] - 0.5) < 1e-2


def test_oracle_dequantizes_the_packed_words(synth):
    rng = np.random.default_rng(1)
    q = rng.integers(0, 256, (5, 128), dtype=np.uint8)
    s = synth.f32_to_bf16_bits(rng.uniform(1e-4, 1e-3, (5, 2)).astype(np.float32))
    b = synth.f32_to_bf16_bits(rng.uniform(-0.1, 0.1, (5, 2)).astype(np.float32))
    packed = q.view(np.uint32)  # element 4i + j in bits 8j..8j+7 of word i (little-endian bytes)
    assert packed[0, 0] == int(q[0, 0]) | int(q[0, 1]) << 8 | int(q[0, 2]) << 16 | int(q[0, 3]) << 24
    got = ora.dequantize_affine8(packed, s, b)
    want = (q.astype(np.float32).reshape(5, 2, 64) * ora.bf16_from_bits(s)[:, :, None]
            + ora.bf16_from_bits(b)[:, :, None]).reshape(5, 128)
    np.testing.assert_array_equal(got, want)


def test_oracle_quantized_model_uses_dequantized_linears(synth, q8_dir, q8_dims):
    q = synth.read_safetensors(os.path.join(q8_dir, "ar-8bit.safetensors"))
    o = ora.OracleAR(q, q8_dims, bf16=True)
    assert "lm_head.scales" not in o.w
    w = o.w["model.layers.0.mlp.down_proj.weight"]
    assert w.dtype == np.float32 and w.shape == (q8_dims.hidden, q8_dims.ffn)
    ref = ora.dequantize_affine8(q["model.layers.0.mlp.down_proj.weight"], q["model.layers.0.mlp.down_proj.scales"],
                                 q["model.layers.0.mlp.down_proj.biases"])
    np.testing.assert_array_equal(w, ref)
    logits, _ = o.prefill([1, 2, 3], 16, None)
    assert logits.shape == (q8_dims.vocab,) and np.all(np.isfinite(logits))


def test_small_widths_cannot_be_group_quantized(synth, tmp_path):
    with pytest.raises(ValueError, match="group-64"):
        synth.write_converted(str(tmp_path / "t"), synth.TINY, workers=1, precisions=("bf16", "8bit"))


def _copy(src, dst):
    shutil.copytree(src, dst)
    return dst


def test_precision_argument(yar, q8_dir):
    for bad, needle in (("fp8", "precision must be"), ("int4", "precision must be")):
        with pytest.raises(yar.YarError) as e:
            yar.ARModel(q8_dir, any_dims=True, precision=bad)
        assert e.value.kind == "ValueError" and needle in e.value.message


@pytest.mark.parametrize("edit,kind,needle", [
    (lambda r: r.clear(), "FileNotFoundError", "does not contain 8bit AR weights"),
    (lambda r: r.update(ar="ar-bf16.safetensors"), "ValueError", "filename does not match"),
    (lambda r: r.update(bits=4), "ValueError", "Invalid affine quantization"),
    (lambda r: r.update(group_size=32), "ValueError", "Invalid affine quantization"),
    (lambda r: r.update(mode="mxfp4"), "ValueError", "Invalid affine quantization"),
    (lambda r: r.update(linear_only=False), "ValueError", "Invalid affine quantization"),
])
def test_q8_manifest_checks(yar, q8_dir, tmp_path, edit, kind, needle):
    d = _copy(q8_dir, tmp_path / "m")
    man = json.load(open(d / "conversion.json"))
    rec = man["precisions"]["8bit"]
    edit(rec)
    if not rec:
        del man["precisions"]["8bit"]
    json.dump(man, open(d / "conversion.json", "w"))
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d), any_dims=True, precision="8bit")
    assert e.value.kind == kind and needle in e.value.message


def _rewrite_header(path, mutate):
    raw = open(path, "rb").read()
    n = int(np.frombuffer(raw[:8], np.uint64)[0])
    header = json.loads(raw[8:8 + n])
    mutate(header)
    new = json.dumps(header).encode()
    new += b" " * ((8 - len(new) % 8) % 8)
    open(path, "wb").write(np.uint64(len(new)).tobytes() + new + raw[8 + n:])


@pytest.mark.parametrize("mutate,needle", [
    (lambda h: h.pop("model.layers.0.mlp.up_proj.scales"), "Missing AR tensor"),
    # BF16 of the same byte size where U32 is required.
    (lambda h: h["lm_head.weight"].update(dtype="BF16", shape=[h["lm_head.weight"]["shape"][0],
                                                             2 * h["lm_head.weight"]["shape"][1]]),
     "Incompatible AR tensor shape/dtype: lm_head.weight"),
    (lambda h: h["model.layers.0.self_attn.q_proj.biases"].update(shape=[128, 8]), "shape/dtype"),
    (lambda h: h.update({"model.embed_tokens.scales": h["lm_head.scales"]}), "Unexpected AR tensor"),
])
def test_q8_tensor_set_checks(yar, q8_dir, tmp_path, mutate, needle):
    d = _copy(q8_dir, tmp_path / "m")
    _rewrite_header(str(d / "ar-8bit.safetensors"), mutate)
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d), any_dims=True, precision="8bit")
    assert e.value.status == yar.INVALID_INPUT and needle in e.value.message


def test_4bit_artifact_and_packing(synth, q8_dir, q8_dims):
    man = json.load(open(os.path.join(q8_dir, "conversion.json")))
    assert man["precisions"]["4bit"] == {"ar": "ar-4bit.safetensors", "bits": 4, "group_size": 64,
                                         "mode": "affine", "linear_only": True, "embedding_dtype": "bfloat16"}
    q4 = synth.read_safetensors(os.path.join(q8_dir, "ar-4bit.safetensors"))
    b = synth.read_safetensors(os.path.join(q8_dir, "ar-bf16.safetensors"))
    name = "model.layers.0.mlp.down_proj"
    w = q4[name + ".weight"]
    assert w.dtype == np.uint32 and w.shape == (q8_dims.hidden, q8_dims.ffn // 8)
    # Element 8i + j in bits 4j..4j+3 of word i.
    q, _, _ = synth.quantize_affine(synth.bf16_bits_to_f32(b[name + ".weight"]), 4)
    assert q.max() <= 15
    word = int(w[3, 5])
    assert [(word >> (4 * j)) & 15 for j in range(8)] == [int(v) for v in q[3, 40:48]]
    deq = ora.dequantize_affine(w, q4[name + ".scales"], q4[name + ".biases"])
    s = synth.bf16_bits_to_f32(q4[name + ".scales"])
    ref = synth.bf16_bits_to_f32(b[name + ".weight"]).reshape(deq.shape[0], -1, 64)
    err = np.abs(deq.reshape(ref.shape) - ref)
    assert np.all(err <= s[:, :, None] * 0.75 + np.abs(synth.bf16_bits_to_f32(q4[name + ".biases"]))[:, :, None] / 128)
    o = ora.OracleAR(q4, q8_dims, bf16=True)
    np.testing.assert_array_equal(o.w[name + ".weight"], deq)


def test_4bit_manifest_and_tensor_checks(yar, q8_dir, tmp_path):
    d = _copy(q8_dir, tmp_path / "m")
    man = json.load(open(d / "conversion.json"))
    man["precisions"]["4bit"]["bits"] = 8
    json.dump(man, open(d / "conversion.json", "w"))
    with pytest.raises(yar.YarError, match="Invalid affine quantization"):
        yar.ARModel(str(d), any_dims=True, precision="4bit")
    d2 = _copy(q8_dir, tmp_path / "m2")
    # An 8-bit-shaped weight where the 4-bit file must hold [out, in / 8].
    _rewrite_header(str(d2 / "ar-4bit.safetensors"),
                    lambda h: h["lm_head.weight"].update(shape=[h["lm_head.weight"]["shape"][0] // 2,
                                                              2 * h["lm_head.weight"]["shape"][1]]))
    with pytest.raises(yar.YarError, match="shape/dtype: lm_head.weight"):
        yar.ARModel(str(d2), any_dims=True, precision="4bit")
