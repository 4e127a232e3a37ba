"""The converted AR layout from an upstream generator checkpoint (`lyra prepare`'s AR side).

``prepare_ar`` partitions the upstream YuE2 generator weights — one BF16 safetensors set
holding the AR decoder and the NAR acoustic model together — into the directory
``ARModel`` loads (native/src/conversion.cpp:203-300, :440-475; conversion.py:596-761):

* ``config.json``: the generator config, checked against the pinned one (the reference's
  ``expected_config``: hidden 2048, 28 layers, 16 / 8 heads of 128, FFN 6144, vocabulary
  184,704, RMSNorm eps 1e-6, RoPE theta 1e6, context 24,576, untied embeddings, VAE latent
  64, BF16 weights);
* ``ar-bf16.safetensors``: the AR tensors (embedding, final norm, LM head, and every
  ``model.layers.*`` tensor without ``.nar_``), bytes copied unchanged;
* ``nar-bf16.safetensors``: every other tensor (the NAR stage's; not used by this engine);
* ``ar-8bit.safetensors`` / ``ar-4bit.safetensors`` when ``precisions`` names "8bit" /
  "4bit": the linears in affine group-64 form (``synth.write_quantized``: the published
  affine scheme; MLX's own
  quantizer, which the reference calls, is not on this machine, so the 8-bit bytes are
  this build's quantization of the same weights, not the reference's);
* ``conversion.json``: the schema-1 manifest with one record per precision and the size
  and SHA-256 of every written file.

The upstream checkpoint is a safetensors file, or a directory holding ``model.safetensors``
or shards listed by ``model.safetensors.index.json``, with ``config.json`` beside it unless
given. ``any_dims`` accepts other self-consistent dims (tests).
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

PINNED_CONFIG = {
    "model_type": "yue2", "architectures": ["YuE2ForCausalLM"], "hidden_size": 2048, "num_hidden_layers": 28,
    "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128, "intermediate_size": 6144,
    "vocab_size": 184704, "rms_norm_eps": 1e-6, "rope_theta": 1000000, "max_position_embeddings": 24576,
    "tie_word_embeddings": False, "latent_type": "vae", "latent_dim": 64, "max_latent_frames": 24576,
    "timestep_shift": 1.0,
}
DTYPE_BYTES = {"BF16": 2, "F16": 2, "F32": 4, "U32": 4, "I64": 8}


def _same(a, b) -> bool:
    if isinstance(a, bool) or isinstance(b, bool):
        return a is b
    if isinstance(a, (int, float)) and isinstance(b, (int, float)):
        return float(a) == float(b)
    return a == b


def validate_config(config: dict, any_dims: bool = False) -> None:
    """conversion.cpp:222-231: the pinned fields and BF16 weights."""
    if not isinstance(config, dict):
        raise ValueError("Generator config must be a JSON object")
    for key, want in PINNED_CONFIG.items():
        if any_dims and key in ("hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                "head_dim", "intermediate_size", "vocab_size", "rope_theta",
                                "max_position_embeddings", "max_latent_frames", "rms_norm_eps"):
            if key not in config:
                raise ValueError(f"Pinned generator config mismatch: {key}")
            continue
        if key not in config or not _same(config[key], want):
            raise ValueError(f"Pinned generator config mismatch: {key}")
    if config.get("dtype", config.get("torch_dtype", "")) != "bfloat16":
        raise ValueError("Pinned generator must declare bfloat16 weights")


def ar_key(name: str) -> bool:
    """conversion.cpp:270-275: the AR partition's tensors."""
    return name in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight") or (
        name.startswith("model.layers.") and ".nar_" not in name)


def _header(path: str):
    with open(path, "rb") as f:
        n = int(np.frombuffer(f.read(8), np.uint64)[0])
        if n < 2 or n > 64 << 20:
            raise ValueError(f"Invalid safetensors header size: {path}")
        h = json.loads(f.read(n))
    size = os.path.getsize(path)
    out = {}
    for name, rec in h.items():
        if name == "__metadata__":
            continue
        b, e = rec["data_offsets"]
        nbytes = DTYPE_BYTES.get(rec["dtype"], 0) * int(np.prod(rec["shape"], dtype=np.int64))
        if rec["dtype"] not in DTYPE_BYTES or e - b != nbytes or 8 + n + e > size:
            raise ValueError(f"Truncated or inconsistent safetensors tensor: {name}")
        out[name] = dict(rec, path=path, start=8 + n + b)
    return out


def _sources(src: str):
    """{name: record} over the upstream file(s) and the directory holding them."""
    if os.path.isfile(src):
        return _header(src), os.path.dirname(os.path.abspath(src))
    index = os.path.join(src, "model.safetensors.index.json")
    files = []
    if os.path.exists(index):
        files = sorted(set(json.load(open(index))["weight_map"].values()))
    elif os.path.exists(os.path.join(src, "model.safetensors")):
        files = ["model.safetensors"]
    if not files:
        raise FileNotFoundError(f"No upstream safetensors in {src}")
    recs = {}
    for f in files:
        for name, rec in _header(os.path.join(src, f)).items():
            if name in recs:
                raise ValueError(f"Duplicate upstream tensor: {name}")
            recs[name] = rec
    return recs, src


def _write(path: str, recs: dict, names: list, metadata: dict) -> dict:
    header, off = {}, 0
    for name in names:
        r = recs[name]
        n = DTYPE_BYTES[r["dtype"]] * int(np.prod(r["shape"], dtype=np.int64))
        header[name] = {"dtype": r["dtype"], "shape": list(r["shape"]), "data_offsets": [off, off + n]}
        off += n
    header["__metadata__"] = metadata
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "xb") as out:
        out.write(np.uint64(len(raw)).tobytes() + raw)
        for name in names:
            r = recs[name]
            left = header[name]["data_offsets"][1] - header[name]["data_offsets"][0]
            with open(r["path"], "rb") as f:
                f.seek(r["start"])
                while left:
                    chunk = f.read(min(left, 64 << 20))
                    if not chunk:
                        raise ValueError(f"Source tensor ended unexpectedly: {name}")
                    out.write(chunk)
                    left -= len(chunk)
        out.flush()
        os.fsync(out.fileno())
    return file_record(path)


def _synth():
    """synth.py beside this file (the package directory's name is not importable)."""
    import sys
    from importlib import util
    name = "yue2_mlx_b200_synth"
    if name not in sys.modules:
        spec = util.spec_from_file_location(name, os.path.join(os.path.dirname(os.path.abspath(__file__)), "synth.py"))
        mod = util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def file_record(path: str) -> dict:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(64 << 20), b""):
            h.update(chunk)
    return {"bytes": os.path.getsize(path), "sha256": h.hexdigest()}


def prepare_ar(src: str, out_dir: str, precisions=("bf16",), config: dict | None = None,
               any_dims: bool = False) -> str:
    """Write the converted AR directory (see the module docstring); returns ``out_dir``."""
    if "bf16" not in precisions or any(p not in ("bf16", "8bit", "4bit") for p in precisions):
        raise ValueError("precisions: 'bf16', optionally with '8bit' and '4bit'")
    recs, base = _sources(src)
    if config is None:
        cpath = os.path.join(base, "config.json")
        if not os.path.exists(cpath):
            raise FileNotFoundError(f"Missing generator config: {cpath}")
        config = json.load(open(cpath))
    validate_config(config, any_dims)
    bad = [n for n, r in recs.items() if r["dtype"] != "BF16"]
    if bad:
        raise ValueError(f"Upstream tensors must be BF16: {bad[0]}")
    # The AR tensor set the loader requires, in its canonical order (synth.tensor_specs).
    synth = _synth()
    dims = synth.Dims(hidden=config["hidden_size"], layers=config["num_hidden_layers"],
                      heads=config["num_attention_heads"], kv_heads=config["num_key_value_heads"],
                      head_dim=config["head_dim"], ffn=config["intermediate_size"], vocab=config["vocab_size"],
                      eps=float(config["rms_norm_eps"]), theta=float(config["rope_theta"]),
                      context=config.get("max_position_embeddings", 24576))
    ar_names = []
    for name, shape in synth.tensor_specs(dims):
        if name not in recs:
            raise ValueError(f"Missing partition tensors: {name}")
        if tuple(recs[name]["shape"]) != tuple(shape):
            raise ValueError(f"Incompatible upstream tensor shape: {name}")
        ar_names.append(name)
    extra = [n for n in recs if ar_key(n) and n not in set(ar_names)]
    if extra:
        raise ValueError(f"Unexpected AR tensor: {extra[0]}")
    nar_names = sorted((n for n in recs if not ar_key(n)), key=lambda n: (recs[n]["path"], recs[n]["start"]))
    os.makedirs(out_dir, exist_ok=True)
    files = {"ar-bf16.safetensors": _write(os.path.join(out_dir, "ar-bf16.safetensors"), recs, ar_names,
                                           {"format": "mlx", "partition": "ar", "precision": "bfloat16"})}
    if nar_names:
        files["nar-bf16.safetensors"] = _write(os.path.join(out_dir, "nar-bf16.safetensors"), recs, nar_names,
                                               {"format": "mlx", "partition": "nar", "precision": "bfloat16"})
    manifest_precisions = {"bf16": {"ar": "ar-bf16.safetensors", "nar": "nar-bf16.safetensors",
                                    "dtype": "bfloat16"}}
    for bits in (8, 4):
        if f"{bits}bit" in precisions:
            synth.write_quantized(out_dir, dims, bits=bits)
            files[f"ar-{bits}bit.safetensors"] = file_record(os.path.join(out_dir, f"ar-{bits}bit.safetensors"))
            manifest_precisions[f"{bits}bit"] = synth.quantized_record(bits)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    files["config.json"] = file_record(os.path.join(out_dir, "config.json"))
    manifest = {"schema": 1, "format": "lyra-yue2-mlx",
                "source": {"upstream": os.path.abspath(src)}, "upstream": "yue2", "conversion": "yue2-mlx_b200",
                "precisions": manifest_precisions, "files": files}
    with open(os.path.join(out_dir, "conversion.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return out_dir
