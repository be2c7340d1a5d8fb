"""The checkpoint converter's write contract on CPU (no GPU work: quantized tensors come from stand-in producers).

Covers the parts of the contract in ``comfy_quant_bench_b200/convert.py``: the refusals (source == output,
existing output / manifest, already-quantized source, stale partial), the planned header (safetensors reads the
file back), byte-for-byte copies of unselected tensors, the manifest placed with the model, and a failed write
leaving neither the model nor a partial behind.
"""
import json
from pathlib import Path

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

from comfy_quant_bench_b200 import convert as C
from comfy_quant_bench_b200 import formats as F


def _source(tmp: Path, metadata=None, extra=None) -> Path:
    g = torch.Generator().manual_seed(0)
    t = {"blocks.0.attn.qkv.weight": torch.randn(768, 512, generator=g).to(torch.bfloat16),
         "blocks.0.attn.qkv.bias": torch.randn(768, generator=g).to(torch.bfloat16),
         "blocks.0.norm.weight": torch.randn(512, generator=g),
         "blocks.0.mlp.fc1.weight": torch.randn(1024, 512, generator=g).to(torch.float16),
         "blocks.0.mlp.fc2.weight": torch.randn(512, 1000, generator=g),          # K=1000: no format accepts it
         "pos_embed": torch.randn(4, 512, generator=g)}
    t.update(extra or {})
    p = tmp / "model.safetensors"
    save_file(t, str(p), metadata=metadata or {"modelspec.title": "test"})
    return p


def _stand_in_entries(conv, selected, fmt):
    """Entries planned like convert.plan, with zero tensors of the planned dtype/shape standing in for the
    GPU-quantized ones."""
    entries = []
    for name, info in sorted(conv.header.items(), key=lambda kv: kv[1]["data_offsets"][0]):
        if name in selected:
            for key, dtype, shape in fmt.tensors(name, list(info["shape"])):
                n = C.DTYPE_BYTES[dtype]
                for d in shape:
                    n *= d
                entries.append(C.Entry(key, dtype, shape, n,
                                       produce=lambda dt=dtype, sh=shape: torch.zeros(sh, dtype=C.TORCH_OF[dt])))
        else:
            s, e = info["data_offsets"]
            entries.append(C.Entry(name, info["dtype"], list(info["shape"]), e - s, copy=(s, e - s)))
    return entries


def test_select_layers_by_format_and_regex(tmp_path):
    conv = C.Conversion(_source(tmp_path), tmp_path / "out.safetensors")
    fmt = F.AffineW4A8()
    assert C.select_layers(conv.header, fmt, None, None) == ["blocks.0.attn.qkv.weight", "blocks.0.mlp.fc1.weight"]
    assert C.select_layers(conv.header, fmt, "mlp", None) == ["blocks.0.mlp.fc1.weight"]
    assert C.select_layers(conv.header, fmt, None, "qkv") == ["blocks.0.mlp.fc1.weight"]


def test_commit_writes_a_loadable_checkpoint_and_manifest(tmp_path):
    src = _source(tmp_path)
    out = tmp_path / "out.safetensors"
    conv = C.Conversion(src, out)
    conv.refuse_unsafe()
    fmt = F.AffineW4A8()
    selected = C.select_layers(conv.header, fmt, None, None)
    meta = F.quant_metadata(conv.metadata, F.layer_configs({n: fmt for n in selected}), fmt.name)
    written = conv.commit(_stand_in_entries(conv, selected, fmt), meta, lambda: {"quantization": fmt.name})
    assert out.exists() and conv.sidecar.exists()
    assert not conv.partial.exists() and not conv.sidecar_partial.exists()
    assert out.stat().st_size == conv.output_size and written > 0
    with safe_open(str(out), "pt") as f, safe_open(str(src), "pt") as s:
        md = f.metadata()
        assert md["modelspec.title"] == "test" and md["quantization"] == "affine_w4a8"
        layers = json.loads(md["_quantization_metadata"])["layers"]
        assert set(layers) == {"blocks.0.attn.qkv", "blocks.0.mlp.fc1"}
        assert F.format_from_config(layers["blocks.0.attn.qkv"]) == fmt
        assert f.get_tensor("blocks.0.attn.qkv.weight").shape == (768, 256)
        assert f.get_tensor("blocks.0.attn.qkv.weight_scale").dtype == torch.bfloat16
        assert f.get_tensor("blocks.0.attn.qkv.weight_zeros").shape == (4, 768)
        for name in ("blocks.0.attn.qkv.bias", "blocks.0.norm.weight", "blocks.0.mlp.fc2.weight", "pos_embed"):
            assert torch.equal(f.get_tensor(name), s.get_tensor(name)), name
    assert json.loads(conv.sidecar.read_text())["quantization"] == "affine_w4a8"


@pytest.mark.parametrize("case", ["same_path", "existing_output", "existing_manifest", "quantized_metadata",
                                  "inline_marker", "stale_partial"])
def test_refusals(tmp_path, case):
    extra = {"blocks.0.attn.qkv.comfy_quant": torch.zeros(3, dtype=torch.uint8)} if case == "inline_marker" else None
    md = {"_quantization_metadata": "{}"} if case == "quantized_metadata" else None
    src = _source(tmp_path, metadata=md, extra=extra)
    out = src if case == "same_path" else tmp_path / "out.safetensors"
    conv = C.Conversion(src, out)
    if case == "existing_output":
        out.write_bytes(b"x")
    if case == "existing_manifest":
        conv.sidecar.write_text("{}")
    if case == "stale_partial":
        conv.partial.write_bytes(b"x")
    with pytest.raises(SystemExit):
        conv.refuse_unsafe()


def test_failed_write_leaves_no_model_and_no_partial(tmp_path):
    src = _source(tmp_path)
    out = tmp_path / "out.safetensors"
    conv = C.Conversion(src, out)
    fmt = F.AffineW4A8()
    selected = C.select_layers(conv.header, fmt, None, None)
    entries = _stand_in_entries(conv, selected, fmt)
    bad = next(e for e in entries if e.produce is not None)
    bad.produce = lambda: torch.zeros(3, dtype=torch.int8)            # not the planned shape
    with pytest.raises(RuntimeError):
        conv.commit(entries, {}, lambda: {})
    assert not out.exists() and not conv.partial.exists() and not conv.sidecar.exists()
    assert not conv.sidecar_partial.exists()


def test_cli_dry_run_and_cpu_refusal(tmp_path, capsys):
    src = _source(tmp_path)
    assert C.main(["--input", str(src), "--format", "convrot_w4a4", "--dry-run"]) == 0
    assert "Selected linear weights: 2" in capsys.readouterr().out
    if not torch.cuda.is_available():
        with pytest.raises(SystemExit, match="CUDA is unavailable"):
            C.main(["--input", str(src), "--format", "affine_w4a8"])
        assert not (tmp_path / "model_affine_w4a8.safetensors").exists()
