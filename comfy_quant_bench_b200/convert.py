"""Checkpoint converter: a high-precision ``.safetensors`` model -> a quantized ``.safetensors`` in one of the packed
formats of ``formats.py``, the weights rotated and quantized by the library's weight kernel on the GPU.

    python -m comfy_quant_bench_b200.convert --input model.safetensors --format affine_w4a8 \\
        [--output OUT] [--group-size G] [--convrot-groupsize R] [--layers REGEX] [--exclude REGEX] [--dry-run]

Formats: affine_w4a8 (awq tensors, group 128, optional ConvRot; the W4A8 affine linear), convrot_w4a4 (rotated
per-row int4, the ConvRot W4A4 linear), int8_tensorwise (W8A8, optional ConvRot), awq_w4a16.  Selected layers: every
2-D floating-point ``*.weight`` the format accepts, narrowed by ``--layers`` / ``--exclude``; every other tensor is
copied byte for byte.  The output's ``__metadata__`` carries the source's keys plus ``_quantization_metadata``
(format version and one entry per layer) and ``quantization``; a ``<output>.quant.json`` manifest sits beside it.

The write follows the checkpoint contract of comfy-quant-bench's converters (``tools/_conversion.py:4-13``):

 1. refuse source == output, and an existing output or manifest;
 2. refuse a source that is already quantized (``_quantization_metadata`` in its metadata, or inline
    ``.comfy_quant`` tensors);
 3. refuse a stale ``<output>.partial``;
 4. plan the whole header, every ``data_offsets``, before writing a byte (the quantized shapes are analytic);
 5. stream the tensors in source order, one at a time: quantized on the GPU, or copied from the source file;
 6. check the bytes written against the plan;
 7. write to ``<output>.partial`` opened exclusively, flush, fsync, then put the manifest in place and the model
    after it, removing the partial files in ``finally`` (a crash leaves at most an orphan manifest, never a model
    without one);
 8. refuse when the destination lacks the output size plus 1 GiB of free disk.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil
import struct
import sys
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import torch

from . import formats as F

GIB = 1024 ** 3
CHUNK = 16 * 1024 ** 2
DTYPE_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "I16": 2, "U16": 2, "F16": 2, "BF16": 2,
               "I32": 4, "U32": 4, "F32": 4, "I64": 8, "U64": 8, "F64": 8}
TORCH_OF = {"I8": torch.int8, "U8": torch.uint8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64,
            "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64}
HEADER_OF = {v: k for k, v in TORCH_OF.items()}
FLOAT_DTYPES = ("F16", "BF16", "F32")


# ---------------------------------------------------------------- reading

def read_header(path: Path) -> tuple[dict, dict, int]:
    """(tensor entries, __metadata__, byte offset of the data section) without reading any tensor data."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    metadata = header.pop("__metadata__", {}) or {}
    return header, metadata, 8 + n


def read_tensor(path: Path, data_start: int, info: dict) -> torch.Tensor:
    start, end = info["data_offsets"]
    with open(path, "rb") as f:
        f.seek(data_start + start)
        raw = bytearray(f.read(end - start))
    dt = TORCH_OF[info["dtype"]]
    t = torch.frombuffer(raw, dtype=dt) if raw else torch.empty(0, dtype=dt)
    return t.reshape(info["shape"])


# ---------------------------------------------------------------- the write contract

@dataclass
class Entry:
    """One output tensor: its header fields and where its bytes come from (a copy range or a producer)."""
    key: str
    dtype: str
    shape: list[int]
    nbytes: int
    copy: tuple[int, int] | None = None                         # (offset in the source data section, size)
    produce: Callable[[], torch.Tensor] | None = None


def header_blob(entries: list[Entry], metadata: dict) -> tuple[bytes, int]:
    """The serialized header (8-byte aligned, as safetensors pads it) and the planned data size."""
    hdr, off = {}, 0
    if metadata:
        hdr["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for e in entries:
        hdr[e.key] = {"dtype": e.dtype, "shape": list(e.shape), "data_offsets": [off, off + e.nbytes]}
        off += e.nbytes
    blob = json.dumps(hdr, separators=(",", ":")).encode("utf-8")
    blob += b" " * ((-len(blob)) % 8)
    return blob, off


def tensor_bytes(t: torch.Tensor) -> memoryview:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return memoryview(t.numpy()).cast("B")


class Conversion:
    def __init__(self, source: Path, output: Path):
        self.source, self.output = source, output
        self.sidecar = output.with_suffix(".quant.json")
        self.partial = output.with_name(output.name + ".partial")
        self.sidecar_partial = self.sidecar.with_name(self.sidecar.name + ".partial")
        self.header, self.metadata, self.data_start = read_header(source)
        self.output_size = 0

    def refuse_unsafe(self) -> None:
        """Contract parts 1-3."""
        if self.output == self.source:
            raise SystemExit("Refusing to overwrite the source model")
        if self.output.exists():
            raise SystemExit(f"Refusing to overwrite existing output: {self.output}")
        if self.sidecar.exists():
            raise SystemExit(f"Refusing to overwrite existing manifest: {self.sidecar}")
        if self.metadata.get("_quantization_metadata"):
            raise SystemExit("Refusing to requantize a checkpoint that already has quantization metadata")
        inline = sum(1 for name in self.header if name.endswith(".comfy_quant"))
        if inline:
            raise SystemExit(f"Refusing to requantize: the source carries {inline} inline '.comfy_quant' markers")
        if self.partial.exists():
            raise SystemExit(f"Refusing to overwrite stale partial output: {self.partial}")

    def guard_disk(self, needed: int, headroom_gib: float = 1.0) -> None:
        """Contract part 8."""
        free = shutil.disk_usage(self.output.parent).free
        need = needed + int(headroom_gib * GIB)
        if free < need:
            raise SystemExit(f"Insufficient disk space at {self.output.parent}: need {need} bytes "
                             f"({needed} of output plus {headroom_gib:.0f} GiB), free {free}")

    def commit(self, entries: list[Entry], metadata: dict, manifest: Callable[[], dict],
               progress: Callable[[int, int, str], None] | None = None) -> int:
        """Contract parts 4-7.  Returns the data bytes written."""
        blob, planned = header_blob(entries, metadata)
        self.output_size = 8 + len(blob) + planned
        written = 0
        side_created = side_placed = False
        out = open(self.partial, "xb")            # exclusive: never clobbers another writer's partial
        try:
            with open(self.source, "rb") as src, out:
                out.write(struct.pack("<Q", len(blob)))
                out.write(blob)
                for i, e in enumerate(entries, 1):
                    if e.copy is not None:
                        start, size = e.copy
                        src.seek(self.data_start + start)
                        left = size
                        while left:
                            chunk = src.read(min(CHUNK, left))
                            if not chunk:
                                raise RuntimeError(f"source ended early while copying {e.key}")
                            out.write(chunk)
                            left -= len(chunk)
                        written += size
                    else:
                        t = e.produce()
                        if HEADER_OF.get(t.dtype) != e.dtype or list(t.shape) != list(e.shape):
                            raise RuntimeError(f"{e.key}: produced {HEADER_OF.get(t.dtype)} {list(t.shape)}, "
                                               f"planned {e.dtype} {e.shape}")
                        buf = tensor_bytes(t)
                        if len(buf) != e.nbytes:
                            raise RuntimeError(f"{e.key}: {len(buf)} bytes, planned {e.nbytes}")
                        out.write(buf)
                        written += len(buf)
                    if progress:
                        progress(i, len(entries), e.key)
                if written != planned:
                    raise RuntimeError(f"length mismatch: wrote {written} bytes, planned {planned}")
                out.flush()
                os.fsync(out.fileno())
            text = json.dumps(manifest(), indent=2, sort_keys=True) + "\n"
            with open(self.sidecar_partial, "xb") as sp:
                side_created = True
                sp.write(text.encode("utf-8"))
                sp.flush()
                os.fsync(sp.fileno())
            if self.sidecar.exists():
                raise SystemExit(f"Refusing to overwrite existing manifest: {self.sidecar}")
            os.replace(self.sidecar_partial, self.sidecar)
            side_placed = True
            if self.output.exists():                 # checked again here: os.replace overwrites
                raise SystemExit(f"Refusing to overwrite existing output: {self.output}")
            os.replace(self.partial, self.output)
            side_placed = False
        finally:
            if self.partial.exists():
                self.partial.unlink()
            if side_created and self.sidecar_partial.exists():
                self.sidecar_partial.unlink()
            if side_placed and self.sidecar.exists():
                self.sidecar.unlink()
        return written


# ---------------------------------------------------------------- planning

def make_format(name: str, group_size: int | None, convrot_groupsize: int | None) -> F.QuantFormat:
    if name == F.AffineW4A8.name:
        return F.AffineW4A8(group_size=group_size or 128, convrot_groupsize=convrot_groupsize or 0)
    if name == F.ConvrotW4A4.name:
        return F.ConvrotW4A4(convrot_groupsize=convrot_groupsize or 256)
    if name == F.Int8Tensorwise.name:
        return F.Int8Tensorwise(convrot=bool(convrot_groupsize), convrot_groupsize=convrot_groupsize or 256)
    if name == F.AwqW4A16.name:
        return F.AwqW4A16(group_size=group_size or 128)
    raise SystemExit(f"format {name!r} has no weight kernel here (choose one of affine_w4a8, convrot_w4a4, "
                     "int8_tensorwise, awq_w4a16)")


def select_layers(header: dict, fmt, include: str | None, exclude: str | None) -> list[str]:
    inc = re.compile(include) if include else None
    exc = re.compile(exclude) if exclude else None
    out = []
    for name, info in header.items():
        if not name.endswith(".weight") or info["dtype"] not in FLOAT_DTYPES or len(info["shape"]) != 2:
            continue
        if inc and not inc.search(name):
            continue
        if exc and exc.search(name):
            continue
        if fmt.accepts(list(info["shape"])):
            out.append(name)
    return out


def plan(conv: Conversion, selected: list[str], fmt, device) -> list[Entry]:
    """Output entries in source order; a selected layer becomes the format's tensors, produced on the GPU when the
    writer reaches them (one layer in memory at a time; each layer is quantized once for all its tensors)."""
    chosen = set(selected)
    cache: dict[str, list[torch.Tensor]] = {}

    def producer(name: str, idx: int, last: bool):
        def run() -> torch.Tensor:
            if name not in cache:
                w = read_tensor(conv.source, conv.data_start, conv.header[name]).to(device=device, dtype=torch.float32)
                cache.clear()
                cache[name] = fmt.quantize(w)[0]
            t = cache[name][idx]
            if last:
                cache.pop(name, None)
            return t
        return run

    entries = []
    for name, info in sorted(conv.header.items(), key=lambda kv: kv[1]["data_offsets"][0]):
        if name in chosen:
            outs = fmt.tensors(name, list(info["shape"]))
            for i, (key, dtype, shape) in enumerate(outs):
                n = DTYPE_BYTES[dtype]
                for d in shape:
                    n *= d
                entries.append(Entry(key, dtype, shape, n, produce=producer(name, i, i == len(outs) - 1)))
        else:
            start, end = info["data_offsets"]
            entries.append(Entry(name, info["dtype"], list(info["shape"]), end - start, copy=(start, end - start)))
    return entries


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--input", required=True, type=Path)
    ap.add_argument("--output", type=Path)
    ap.add_argument("--format", default=F.AffineW4A8.name,
                    choices=[F.AffineW4A8.name, F.ConvrotW4A4.name, F.Int8Tensorwise.name, F.AwqW4A16.name])
    ap.add_argument("--group-size", type=int)
    ap.add_argument("--convrot-groupsize", type=int)
    ap.add_argument("--layers", help="regex: quantize only matching weight names")
    ap.add_argument("--exclude", help="regex: keep matching weight names in high precision")
    ap.add_argument("--dry-run", action="store_true")
    args = ap.parse_args(argv)

    source = args.input.resolve()
    if not source.is_file() or source.suffix.lower() != ".safetensors":
        raise SystemExit("Input must be an existing .safetensors file")
    output = (args.output or source.with_name(f"{source.stem}_{args.format}.safetensors")).resolve()
    conv = Conversion(source, output)
    conv.refuse_unsafe()
    fmt = make_format(args.format, args.group_size, args.convrot_groupsize)
    selected = select_layers(conv.header, fmt, args.layers, args.exclude)
    if not selected:
        raise SystemExit(f"no weight of {source.name} is accepted by {fmt.name} (with the given --layers/--exclude)")
    print(f"Source: {source}\nFormat: {fmt.layer_config()}\nSelected linear weights: {len(selected)}\n"
          f"Output: {output}")
    if args.dry_run:
        for name in selected[:10]:
            print(f"  {name}: {conv.header[name]['shape']} {conv.header[name]['dtype']}")
        if len(selected) > 10:
            print(f"  ... {len(selected) - 10} more")
        return 0
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is unavailable: the weight kernel runs on the GPU (there is no CPU path)")
    started = time.perf_counter()
    entries = plan(conv, selected, fmt, torch.device("cuda"))
    metadata = F.quant_metadata(conv.metadata, F.layer_configs({n: fmt for n in selected}), fmt.name)
    blob, planned = header_blob(entries, metadata)
    conv.guard_disk(8 + len(blob) + planned)

    def manifest() -> dict:
        return {"source": str(source), "source_size": source.stat().st_size, "output": str(output),
                "output_size": conv.output_size, "quantization": fmt.name, "layer_config": fmt.layer_config(),
                "quantized_tensors": len(selected), "preserved_tensors": len(conv.header) - len(selected),
                "torch_version": torch.__version__, "cuda_version": torch.version.cuda,
                "gpu": torch.cuda.get_device_name(0), "conversion_seconds": round(time.perf_counter() - started, 3)}

    def progress(i: int, n: int, key: str) -> None:
        if i % 64 == 0 or i == n:
            print(f"[{i}/{n}] {key}", flush=True)

    conv.commit(entries, metadata, manifest, progress)
    print(f"Wrote {output} ({conv.output_size} bytes) in {time.perf_counter() - started:.1f} s\nWrote {conv.sidecar}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
