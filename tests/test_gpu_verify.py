"""GPU checkpoint verification (slimdit/verify.py, the reference's tools/verify_checkpoint.py):
distances reduced on the device against numpy recomputations, a self-comparison with zero
findings, a reordered gated projection caught as a finding, and the official-weight mode."""

import struct

import numpy as np
import pytest
import torch

import oracle
import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def converted(tmp_path_factory, golden_meta):
    from slimdit.convert import convert
    case = golden_meta["convert"]["case"]
    d = tmp_path_factory.mktemp("verify")
    src = synthetic.official_checkpoint(d / "official", **case)
    out = d / "ours.safetensors"
    convert(src, out, rank=8, grid=65)
    return src, out


def _tensor_range(path, name):
    raw = path.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    import json
    header = json.loads(raw[8:8 + n])
    b0, b1 = header[name]["data_offsets"]
    return raw, 8 + n + b0, 8 + n + b1, header[name]


def test_self_comparison_has_no_findings(cuda, converted, capsys):
    from slimdit import verify
    from slimdit.safetensors_io import ShardSet
    _, out = converted
    s = ShardSet(out)
    assert verify.compare_reference(s, s, 0.02, 5) == 0
    assert "0 findings" in capsys.readouterr().out


def test_swapped_gated_projection_is_a_finding(cuda, converted, tmp_path, capsys):
    from slimdit import verify
    from slimdit.safetensors_io import ShardSet
    _, out = converted
    key = "blocks.0.mlp.fc1.weight"
    raw, lo, hi, meta = _tensor_range(out, key)
    rows, cols = meta["shape"]
    q = np.frombuffer(raw[lo:hi], dtype=np.int8).reshape(rows, cols)
    _, slo, shi, _ = _tensor_range(out, "blocks.0.mlp.fc1.weight_scale")
    sc = np.frombuffer(raw[slo:shi], dtype=np.float32).reshape(rows)
    half = rows // 2
    q_sw = np.concatenate([q[half:], q[:half]])
    s_sw = np.concatenate([sc[half:], sc[:half]])
    bad = bytearray(raw)
    bad[lo:hi] = q_sw.tobytes()
    bad[slo:shi] = s_sw.tobytes()
    badp = tmp_path / "swapped.safetensors"
    badp.write_bytes(bytes(bad))
    findings = verify.compare_reference(ShardSet(badp), ShardSet(out), 0.02, 5)
    text = capsys.readouterr().out
    # the codes and their row scales are both reordered: two findings, as the reference reports
    assert findings == 2 and "[FAIL]" in text and key in text and "blocks.0.mlp.fc1.weight_scale" in text
    # the device distance equals the numpy one on the rotated-basis values
    a = q_sw.astype(np.float32) * s_sw.reshape(-1, 1)
    b = q.astype(np.float32) * sc.reshape(-1, 1)
    want = np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64))
    dev = torch.device("cuda", 0)
    d = verify._Distances(dev, 1)
    d.int8(0, torch.from_numpy(q_sw).to(dev), torch.from_numpy(s_sw).to(dev), torch.from_numpy(q.copy()).to(dev),
           torch.from_numpy(sc.copy()).to(dev))
    got = float(d.values()[0])
    assert abs(got - want) <= 1e-9 * want


def test_official_mode_matches_numpy(cuda, converted, capsys):
    from slimdit import verify
    from slimdit.safetensors_io import ShardSet
    src, out = converted
    slim, off = ShardSet(out), ShardSet(src)
    layers = ["blocks.0.attn.qkv_proj.weight", "blocks.0.mlp.fc1.weight", "blocks.1.mlp.fc2.weight"]
    errs = verify.official_quant_errors(slim, off, layers)
    for key in layers:
        block, suffix = key.split(".")[1], key.split(".", 2)[2]
        parts = [off.get(f"transformer_blocks.{block}.{n}").float().numpy() for n in verify.OFFICIAL_FOR[suffix]]
        ref = np.concatenate(parts) if len(parts) > 1 else parts[0]
        if suffix == "mlp.fc1.weight":
            h = ref.shape[0] // 2
            ref = np.concatenate([ref[h:], ref[:h]])
        restored = oracle.dequantize_convrot_weight(slim.get(key).numpy(), slim.get(key[:-7] + ".weight_scale").numpy())
        want = np.linalg.norm(restored.astype(np.float64) - ref) / np.linalg.norm(ref.astype(np.float64))
        assert abs(errs[key] - want) <= 1e-9 * want, key
        assert 0.001 < errs[key] < 0.05
    assert verify.compare_official(slim, off, layers, 8, 65) == 0
    assert "modulation error" in capsys.readouterr().out


def test_nvfp4_checkpoint_self_comparison(cuda, golden_meta, tmp_path):
    from slimdit import verify
    from slimdit.convert import convert
    from slimdit.safetensors_io import ShardSet
    case = golden_meta["convert"]["case"]
    src = synthetic.official_checkpoint(tmp_path / "official", **case)
    out = tmp_path / "fp4.safetensors"
    convert(src, out, rank=8, grid=65, quant="nvfp4")
    s = ShardSet(out)
    assert verify.compare_reference(s, s, 0.02, 3) == 0
    errs = verify.official_quant_errors(s, ShardSet(src), ["blocks.0.mlp.fc2.weight"])
    assert 0.02 < errs["blocks.0.mlp.fc2.weight"] < 0.2
