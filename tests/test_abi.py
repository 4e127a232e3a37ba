"""The C ABI without a GPU: the library loads, exports every declared entry point, and
the loader's validation (native/src/ar.cpp:133-238) rejects bad checkpoints with the
reference's error types before touching the device."""
import json
import os
import shutil
import threading

import numpy as np
import pytest

from tests.conftest import ROOT, load_package


@pytest.fixture(scope="module")
def yar():
    return load_package()


def test_library_exports_every_declared_function(yar):
    names = yar.header_functions(os.path.join(ROOT, "include", "yue2ar.h"))
    assert len(names) >= 17
    for n in names:
        assert hasattr(yar.lib, n), n
    assert yar.lib.yar_version().decode().startswith("yue2ar-cuda")


def test_missing_directory_is_file_not_found(yar, tmp_path):
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(tmp_path / "nope"))
    assert e.value.status == yar.INVALID_INPUT and e.value.kind == "FileNotFoundError"


def _copy(src, dst):
    shutil.copytree(src, dst)
    return dst


def test_pinned_config_is_enforced(yar, tiny_dir, tmp_path):
    d = _copy(tiny_dir, tmp_path / "m")
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d))  # tiny dims are not the pinned YuE2-3B config
    assert e.value.kind == "ValueError" and "Incompatible YuE2 config" in e.value.message


@pytest.mark.parametrize("edit,needle", [
    (lambda c: c.update(tie_word_embeddings=True), "untied"),
    (lambda c: c.update(rope_scaling={"type": "linear"}), "RoPE"),
    (lambda c: c.update(hidden_act="gelu"), "silu"),
    (lambda c: c.update(rms_norm_eps=-1.0), "rms_norm_eps"),
    (lambda c: c.update(num_hidden_layers=2.5), "positive integer"),
])
def test_config_checks(yar, tiny_dir, tmp_path, edit, needle):
    d = _copy(tiny_dir, tmp_path / "m")
    cfg = json.load(open(d / "config.json"))
    edit(cfg)
    json.dump(cfg, open(d / "config.json", "w"))
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d), any_dims=True)
    assert e.value.status == yar.INVALID_INPUT and needle in e.value.message


def test_manifest_checks(yar, tiny_dir, tmp_path):
    d = _copy(tiny_dir, tmp_path / "m")
    man = json.load(open(d / "conversion.json"))
    man["schema"] = 2
    json.dump(man, open(d / "conversion.json", "w"))
    with pytest.raises(yar.YarError, match="schema-1"):
        yar.ARModel(str(d), any_dims=True)
    man["schema"] = 1
    del man["precisions"]["bf16"]
    json.dump(man, open(d / "conversion.json", "w"))
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d), any_dims=True)
    assert e.value.kind == "FileNotFoundError"


def _rewrite_header(path, mutate):
    raw = open(path, "rb").read()
    n = int(np.frombuffer(raw[:8], np.uint64)[0])
    header = json.loads(raw[8:8 + n])
    mutate(header)
    new = json.dumps(header).encode()
    new += b" " * ((8 - len(new) % 8) % 8)
    # Keep the data section where it was relative to the (possibly longer) header.
    open(path, "wb").write(np.uint64(len(new)).tobytes() + new + raw[8 + n:])


@pytest.mark.parametrize("mutate,needle", [
    (lambda h: h.pop("model.layers.1.mlp.up_proj.weight"), "Missing AR tensor"),
    (lambda h: h.update({"model.layers.0.extra.weight": h["model.norm.weight"]}), "Unexpected AR tensor"),
    (lambda h: h["model.norm.weight"].update(shape=[128, 2]), "shape"),
    (lambda h: h["model.norm.weight"].update(dtype="F16"), "dtype"),
])
def test_tensor_set_checks(yar, tiny_dir, tmp_path, mutate, needle):
    d = _copy(tiny_dir, tmp_path / "m")
    _rewrite_header(str(d / "ar-bf16.safetensors"), mutate)
    with pytest.raises(yar.YarError) as e:
        yar.ARModel(str(d), any_dims=True)
    assert e.value.status == yar.INVALID_INPUT and needle in e.value.message


def test_truncated_file_is_rejected(yar, tiny_dir, tmp_path):
    d = _copy(tiny_dir, tmp_path / "m")
    p = d / "ar-bf16.safetensors"
    size = os.path.getsize(p)
    with open(p, "r+b") as f:
        f.truncate(size - 4096)
    with pytest.raises(yar.YarError, match="Truncated|inconsistent"):
        yar.ARModel(str(d), any_dims=True)


def test_last_error_is_thread_local(yar, tmp_path):
    with pytest.raises(yar.YarError):
        yar.ARModel(str(tmp_path / "missing"))
    seen = []
    t = threading.Thread(target=lambda: seen.append(yar.lib.yar_last_error().decode()))
    t.start()
    t.join()
    assert seen == [""]
    assert "Missing file" in yar.lib.yar_last_error().decode()
