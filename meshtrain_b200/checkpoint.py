"""Checkpoint / resume keyed by global tensor IDs.

Layout::

    <dir>/step-<n>/stage-<s>.safetensors     one file per stage
    <dir>/step-<n>/stage-<s>.json            sidecar: stage, number of stages, layer range
    <dir>/step-<n>/manifest.json             optional: step, all layer ranges, config

Each stage writes its own file and sidecar, so stages on different machines
need no coordination; a step is complete when the sidecars of all its stages
are present.  A rank of an interleaved 1F1B program holds several model chunks;
chunk c of rank r is virtual stage c * S + r of S * chunks, and each chunk is
written as the file of its virtual stage (one contiguous layer range per file).

Tensor names are the global IDs ``model.layers.<g>.<param>`` (fp32 master
weights), ``model.layers.<g>.<param>.optim.exp_avg`` / ``.exp_avg_sq`` (Adam
moments) and ``optim.step.stage<s>``, so a checkpoint written with one stage
split loads into any other: a stage reads the IDs of its own layers from
whichever files hold them.  Resuming continues the deterministic data stream
at ``step`` (``PipelineSettings.step_offset`` for the host runtime, the step
argument of ``PipelineTrainer.step`` for the device engine).

The files use the safetensors layout (8-byte little-endian header length,
JSON header with dtype / shape / byte offsets, then the raw little-endian
tensor bytes), written and read here without extra dependencies; the
reference defines tensor IDs but saves nothing (reference
runtime/tensor_store.py:64-70).
"""

from __future__ import annotations

import json
import os
import struct
from pathlib import Path

import torch

_DT = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.float64: "F64",
       torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
       torch.bool: "BOOL"}
_TD = {v: k for k, v in _DT.items()}


def save_tensors(path: str | Path, tensors: dict[str, torch.Tensor], metadata: dict[str, str] | None = None) -> None:
    """Write ``tensors`` as one safetensors file (atomically: temp file + rename)."""
    header: dict = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        blobs.append(t)
        off += nbytes
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * (-len(raw) % 8)  # keep the data section 8-byte aligned
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for t in blobs:
            if t.numel():
                f.write(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bool else t.numpy().tobytes())
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def read_header(path: str | Path) -> tuple[dict, int]:
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if n > 100 * 1024 ** 2:
            raise ValueError(f"{path}: implausible header length {n}")
        return json.loads(f.read(n)), 8 + n


def load_tensors(path: str | Path, names: set[str] | None = None) -> dict[str, torch.Tensor]:
    """Tensors of one file (only ``names`` when given), read with one seek per tensor."""
    header, base = read_header(path)
    out = {}
    with open(path, "rb") as f:
        for name, info in header.items():
            if name == "__metadata__" or (names is not None and name not in names):
                continue
            b, e = info["data_offsets"]
            f.seek(base + b)
            buf = bytearray(f.read(e - b))
            dt = _TD[info["dtype"]]
            t = torch.frombuffer(buf, dtype=torch.uint8) if buf else torch.empty(0, dtype=torch.uint8)
            out[name] = t.view(dt).reshape(info["shape"]).clone() if buf else torch.empty(info["shape"], dtype=dt)
    return out


def step_dir(root: str | Path, step: int) -> Path:
    return Path(root) / f"step-{step}"


def _sidecars(d: Path) -> list[dict]:
    return [json.loads(p.read_text()) for p in sorted(d.glob("stage-*.json"))]


def complete(d: Path) -> bool:
    """True when every stage of the split that wrote ``d`` has its file and sidecar."""
    cars = _sidecars(d)
    return bool(cars) and len(cars) == cars[0]["num_stages"] and all((d / c["file"]).exists() for c in cars)


def write_manifest(root: str | Path, step: int, *, ranges: list[tuple[int, int]], config: dict | None = None,
                   extra: dict | None = None) -> Path:
    d = step_dir(root, step)
    manifest = {"format": "meshtrain-checkpoint/1", "step": step, "num_stages": len(ranges),
                "stages": [{"stage": i, "layers": list(r), "file": f"stage-{i}.safetensors"}
                           for i, r in enumerate(ranges)], "config": config or {}, **(extra or {})}
    missing = [s["file"] for s in manifest["stages"] if not (d / s["file"]).exists()]
    if missing:
        raise FileNotFoundError(f"checkpoint step {step} is incomplete: {missing}")
    (d / "manifest.json").write_text(json.dumps(manifest, indent=2, default=str))
    return d


def latest_step(root: str | Path) -> int | None:
    """Newest step whose every stage file is present (manifest or per-stage sidecars)."""
    steps = sorted((int(d.name.split("-", 1)[1]) for d in Path(root).glob("step-*")
                    if (d / "manifest.json").exists() or complete(d)), reverse=True)
    return steps[0] if steps else None


def load_for_layers(root: str | Path, step: int, layers: tuple[int, int]) -> dict[str, torch.Tensor]:
    """Every tensor of global layers [start, end) at ``step``, whatever the split it was saved with."""
    d = step_dir(root, step)
    if (d / "manifest.json").exists():
        stages = json.loads((d / "manifest.json").read_text())["stages"]
    else:
        stages = _sidecars(d)
    start, end = layers
    out: dict[str, torch.Tensor] = {}
    covered = set()
    for st in stages:
        a, b = st["layers"]
        if b <= start or a >= end:
            continue
        covered.update(range(max(a, start), min(b, end)))
        header, _ = read_header(d / st["file"])
        want = {n for n in header if n.startswith("model.layers.") and start <= int(n.split(".")[2]) < end}
        out.update(load_tensors(d / st["file"], want))
        steps = load_tensors(d / st["file"], {f"optim.step.stage{st['stage']}"})
        if steps:
            out["optim.step"] = next(iter(steps.values()))
    if covered != set(range(start, end)):
        raise FileNotFoundError(f"checkpoint step {step} lacks layers {sorted(set(range(start, end)) - covered)}")
    return out


def _save_stage_file(root, step: int, stage: int, num_stages: int, layers, tensors: dict) -> Path:
    d = step_dir(root, step)
    path = d / f"stage-{stage}.safetensors"
    save_tensors(path, tensors, {"step": step, "stage": stage, "layers": f"{layers[0]},{layers[1]}"})
    (d / f"stage-{stage}.json").write_text(json.dumps({"stage": stage, "num_stages": num_stages,
                                                       "layers": list(layers), "step": step, "file": path.name}))
    return path


# ------------------------------------------------------------------ device engine
def _global_range(engine, units: tuple[int, int] | None = None) -> tuple[int, int]:
    """The model layers a range of an engine's units belongs to (half-block units share
    their block's index); the engine's whole range by default."""
    a, b = units if units is not None else (engine.start, engine.end)
    g = engine.spec.global_layer
    return g(a), g(b - 1) + 1


def _chunk_files(engine) -> list[tuple[int, int, tuple[int, int]]]:
    """(file index, number of files, unit range) for each model chunk the engine holds.

    A rank with one chunk writes ``stage-<stage>``.  A rank of an interleaved program
    holds chunk c of rank r as virtual stage c * S + r of S * chunks; each chunk is one
    contiguous layer range and gets the file of its virtual stage, so the step is
    complete when every virtual stage has written, and any later split reads it.
    """
    chunks = getattr(engine, "chunks", 1)
    if chunks == 1:
        return [(engine.stage, engine.num_stages, (engine.start, engine.end))]
    total = engine.num_stages * chunks
    return [(c * engine.num_stages + engine.stage, total, tuple(r)) for c, r in enumerate(engine.chunk_ranges)]


def save_stage_checkpoint(root: str | Path, engine, step: int) -> Path:
    """Writes this rank's tensors (one file per model chunk); returns the last file written."""
    sd = engine.state_dict()
    opt_step = sd.pop("optim.step").reshape(1)
    g = engine.spec.global_layer
    path = None
    for index, count, units in _chunk_files(engine):
        lo, hi = _global_range(engine, units)
        # names of the parameters of this chunk's units (a half-block unit holds part of a block)
        owned = {f"model.layers.{g(engine.layer_ids[li])}.{name}" for li, name, *_ in engine.flat.entries
                 if units[0] <= engine.layer_ids[li] < units[1]}
        part = {k: v for k, v in sd.items() if k.split(".optim.")[0] in owned}
        part[f"optim.step.stage{index}"] = opt_step
        path = _save_stage_file(root, step, index, count, (lo, hi), part)
    return path


def load_stage_checkpoint(root: str | Path, engine, step: int | None = None) -> int:
    step = latest_step(root) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no checkpoint under {root}")
    sd: dict[str, torch.Tensor] = {}
    for _index, _count, units in _chunk_files(engine):
        sd.update(load_for_layers(root, step, _global_range(engine, units)))
    sd["optim.step"] = sd.get("optim.step", torch.tensor([0])).reshape(())
    engine.load_state_dict(sd)
    return step


# ------------------------------------------------------------------ host runtime stage
def stage_state(stage) -> dict[str, torch.Tensor]:
    out = {}
    for n, p in stage.module.named_parameters():
        gid = stage.global_name(n)
        out[gid] = p.detach()
        if stage.optimizer is not None:
            for k, v in stage.optimizer.state.get(p, {}).items():
                if torch.is_tensor(v) and v.dim() > 0:
                    out[f"{gid}.optim.{k}"] = v.detach()
                elif k == "step":
                    out[f"optim.step.stage{stage.stage_index}"] = torch.tensor([int(float(v))])
    return out


def save_host_stage(root: str | Path, stage, step: int, layers: tuple[int, int]) -> Path:
    return _save_stage_file(root, step, stage.stage_index, stage.num_stages, layers, stage_state(stage))


def load_host_stage(root: str | Path, stage, layers: tuple[int, int], step: int | None = None) -> int:
    step = latest_step(root) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no checkpoint under {root}")
    sd = load_for_layers(root, step, layers)
    opt_step = int(sd.get("optim.step", torch.tensor([0])).reshape(-1)[0])
    with torch.no_grad():
        for n, p in stage.module.named_parameters():
            gid = stage.global_name(n)
            p.copy_(sd[gid].to(p.dtype))
            if stage.optimizer is not None and f"{gid}.optim.exp_avg" in sd:
                st = stage.optimizer.state[p]
                for k in ("exp_avg", "exp_avg_sq"):
                    st[k] = sd[f"{gid}.optim.{k}"].to(p.device, torch.float32).clone()
                st["step"] = torch.tensor(float(opt_step))
    return step
