"""Checkpoint access for the expert path: the manifest and one-read MXFP4 projections.

The reference maps every checkpoint tensor to (shard file, absolute byte offset, nbytes,
shape, dtype, role) in a gzip'd JSON-lines manifest built from the safetensors headers
(``tools/k3_manifest.py:40-156``), and its ``TensorSource`` reads tensors, row blocks and
expert projections by those records (``air_llm/models/kimi_k3/loader.py:44-266``); a
projection's ``weight_scale`` follows its ``weight_packed`` in the shard, so the pair is
one read. This module keeps those record fields, names and errors; the reads are the
library's ``pread`` reader (``k3_file_read_ranges``: threads, adjacent ranges merged)
into pinned host memory, or ``k3_file_read_to_device`` (a pinned double buffer whose
disk reads overlap the host->device copies) straight into HBM.
"""
from __future__ import annotations

import ctypes
import gzip
import hashlib
import json
import os
import re
import struct
from pathlib import Path
from typing import Iterable, Optional

import torch

from . import _lib as L

LAYER_RE = re.compile(r"\.layers\.(\d+)\.")
EXPERT_RE = re.compile(r"\.experts\.(\d+)\.(w[123])\.(weight_packed|weight_scale)$")
DTYPE_BYTES = {"F32": 4, "BF16": 2, "F16": 2, "U8": 1, "I8": 1, "I32": 4, "I64": 8}
_TORCH = {"F32": torch.float32, "BF16": torch.bfloat16, "F16": torch.float16, "U8": torch.uint8,
          "I8": torch.int8, "I32": torch.int32, "I64": torch.int64}
MOE_KEYS = ("gate.weight", "gate.e_score_correction_bias",
            "routed_expert_down_proj.weight", "routed_expert_up_proj.weight",
            "routed_expert_norm.weight", "shared_experts.gate_proj.weight",
            "shared_experts.up_proj.weight", "shared_experts.down_proj.weight")
MAX_HEADER = 256 * 2 ** 20


# ----------------------------------------------------------------- safetensors / manifest

def _weight_or_last(t):
    return t[-2] if t[-1] == "weight" else t[-1]


# Role of a non-expert tensor: the first rule whose test matches the name decides (the
# manifest's role vocabulary, ``k3_manifest.py:64-83``).
_ROLE_RULES = (
    (lambda n: "shared_experts" in n, lambda t: "shared_expert_" + t[-2]),
    (lambda n: "routed_expert_" in n, _weight_or_last),
    (lambda n: "block_sparse_moe.gate" in n, lambda t: "router_" + t[-1]),
    (lambda n: ".self_attn." in n, lambda t: "attn_" + _weight_or_last(t)),
    (lambda n: ".mlp." in n, lambda t: "dense_mlp_" + t[-2]),
    (lambda n: "res_proj" in n or "res_norm" in n, lambda t: t[-2]),
    (lambda n: n.endswith("layernorm.weight") or n.endswith("norm.weight"), lambda t: "norm"),
    (lambda n: "embed_tokens" in n, lambda t: "embed"),
    (lambda n: "lm_head" in n, lambda t: "lm_head"),
)
_COMPONENTS = (("vision_tower.", "vision"), ("mm_projector.", "projector"), ("language_model.", "text"))


def classify(name: str) -> dict:
    """Component / layer / role / expert of a tensor name: the manifest's fields
    (``k3_manifest.py:40-84``)."""
    comp = next((c for prefix, c in _COMPONENTS if name.startswith(prefix)), "other")
    m = LAYER_RE.search(name)
    d: dict = {"component": comp, "layer": int(m.group(1)) if m else None, "expert": None, "role": None}
    m = EXPERT_RE.search(name)
    if m:
        d.update(expert=int(m.group(1)), role=f"routed_expert_{m.group(2)}", kind=m.group(3))
        return d
    tail = name.split(".")
    d["role"] = next((role(tail) for test, role in _ROLE_RULES if test(name)), None)
    return d


def read_header(shard: Path) -> tuple[dict, int]:
    """(header dict, absolute offset of the data section) of a safetensors shard."""
    shard = Path(shard)
    with shard.open("rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        if n > shard.stat().st_size - 8 or n > MAX_HEADER:
            raise ValueError(f"Invalid safetensors header size: {shard.name}")
        return json.loads(fh.read(n)), 8 + n


def manifest_records(ckpt: Path) -> tuple[dict, list]:
    """(meta, records) for a checkpoint directory: the reference's manifest content."""
    ckpt = Path(ckpt)
    cfg = json.loads((ckpt / "config.json").read_text())
    tcfg = cfg["text_config"]
    gsize = tcfg["quantization_config"]["config_groups"]["group_0"]["weights"]["group_size"]
    shards = sorted(ckpt.glob("model-*.safetensors"))
    lac = tcfg["linear_attn_config"]
    nl = tcfg["num_hidden_layers"]
    meta = {
        "__meta__": True,
        "checkpoint": str(ckpt.resolve()),
        "source_revision": os.environ.get("K3_REVISION"),
        "config_sha256": hashlib.sha256((ckpt / "config.json").read_bytes()).hexdigest(),
        "index_sha256": hashlib.sha256((ckpt / "model.safetensors.index.json").read_bytes()).hexdigest(),
        "num_shards": len(shards),
        "num_hidden_layers": nl,
        "num_experts": tcfg["num_experts"],
        "num_experts_per_token": tcfg["num_experts_per_token"],
        "num_shared_experts": tcfg["num_shared_experts"],
        "hidden_size": tcfg["hidden_size"],
        "routed_expert_hidden_size": tcfg["routed_expert_hidden_size"],
        "moe_intermediate_size": tcfg["moe_intermediate_size"],
        "group_size": gsize,
        # the config's layer lists are 1-indexed
        "mla_layers": sorted(i - 1 for i in lac["full_attn_layers"] if i - 1 < nl),
        "kda_layers": sorted(i - 1 for i in lac["kda_layers"] if i - 1 < nl),
    }
    recs = []
    for shard in shards:
        hdr, base = read_header(shard)
        for name, t in hdr.items():
            if name == "__metadata__":
                continue
            s, e = t["data_offsets"]
            rec = {"name": name, "file": shard.name, "offset": base + s, "nbytes": e - s,
                   "shape": t["shape"], "dtype": t["dtype"], **classify(name)}
            if rec.get("kind") == "weight_packed":
                rec["group_size"] = gsize
                rec["scale_tensor"] = name.replace("weight_packed", "weight_scale")
                rec["logical_shape"] = [rec["shape"][0], rec["shape"][1] * 2]
            recs.append(rec)
    return meta, recs


def build_manifest(ckpt: Path, out: Path) -> int:
    """Writes the manifest (``k3_manifest.py build``); returns the record count."""
    meta, recs = manifest_records(ckpt)
    with gzip.open(out, "wt") as fh:
        fh.write(json.dumps(meta) + "\n")
        for r in recs:
            fh.write(json.dumps(r) + "\n")
    return len(recs)


def load_manifest(path: Path) -> tuple[dict, dict]:
    """(meta, {name: record}) of a manifest file."""
    meta, recs = {}, {}
    try:
        fh = gzip.open(path, "rt")
    except FileNotFoundError:
        raise FileNotFoundError(f"manifest not found: {path} (build it with loader.build_manifest)") from None
    with fh:
        for line in fh:
            r = json.loads(line)
            if r.get("__meta__"):
                meta = r
            else:
                recs[r["name"]] = r
    return meta, recs


# -------------------------------------------------------------------------- reads

def pinned_empty(nbytes: int) -> torch.Tensor:
    return torch.empty(int(nbytes), dtype=torch.uint8, pin_memory=torch.cuda.is_available())


def read_ranges(path: Path, ranges: Iterable[tuple[int, int, int]], threads: int = 8) -> int:
    """pread (offset, nbytes, host address) ranges of one file; returns the bytes read."""
    ranges = list(ranges)
    n = len(ranges)
    offs = (ctypes.c_int64 * n)(*[r[0] for r in ranges])
    nbs = (ctypes.c_int64 * n)(*[r[1] for r in ranges])
    dsts = (ctypes.c_void_p * n)(*[r[2] for r in ranges])
    got = ctypes.c_int64(0)
    L.check(L.load_library().k3_file_read_ranges(str(path).encode(), offs, nbs, n, dsts, threads,
                                                 ctypes.byref(got)), "k3_file_read_ranges")
    return int(got.value)


def read_to_device(path: Path, ranges: Iterable[tuple[int, int, int]], staging: torch.Tensor,
                   stream: Optional[torch.cuda.Stream] = None, threads: int = 8) -> None:
    """pread (offset, nbytes, device address) ranges of one file into HBM through the
    pinned ``staging`` buffer (returns once the copies are done)."""
    ranges = list(ranges)
    n = len(ranges)
    offs = (ctypes.c_int64 * n)(*[r[0] for r in ranges])
    nbs = (ctypes.c_int64 * n)(*[r[1] for r in ranges])
    dsts = (ctypes.c_void_p * n)(*[r[2] for r in ranges])
    s = (stream or torch.cuda.current_stream()).cuda_stream
    L.check(L.load_library().k3_file_read_to_device(str(path).encode(), offs, nbs, n, dsts, staging.data_ptr(),
                                                    staging.numel(), threads, s), "k3_file_read_to_device")


class TensorSource:
    """Tensors of a checkpoint by manifest record (the reference's ``TensorSource``,
    ``loader.py:44-266``, for the MoE path): ``raw``, ``tensor``, ``rows``,
    ``row_block``, ``expert_source`` and the layer's dense MoE weights. Host results
    live in pinned memory (ready for asynchronous copies); byte counters as in the
    reference (``bytes_read``, ``expert_bytes``, ``experts_loaded``)."""

    def __init__(self, manifest: Path = Path(os.environ.get("K3_MANIFEST", "manifest.jsonl.gz")),
                 ckpt: Optional[Path] = None, threads: int = 8):
        self.meta, self.recs = load_manifest(Path(manifest))
        self.ckpt = Path(ckpt or os.environ.get("K3_CKPT") or self.meta["checkpoint"])
        self.threads = threads
        self.bytes_read = 0
        self.expert_bytes = 0
        self.experts_loaded = 0

    def reset_counters(self) -> None:
        self.bytes_read = 0
        self.expert_bytes = 0
        self.experts_loaded = 0

    def _locate(self, name: str) -> tuple[Path, int, dict]:
        r = self.recs[name]
        return self.ckpt / r["file"], int(r["offset"]), r

    @staticmethod
    def _view(buf: torch.Tensor, r: dict, shape=None) -> torch.Tensor:
        return buf.view(_TORCH[r["dtype"]]).reshape(list(r["shape"] if shape is None else shape))

    def raw(self, name: str) -> tuple[torch.Tensor, str]:
        """(pinned host tensor in the stored dtype — bf16 as ``torch.bfloat16`` — , dtype
        string) of a whole tensor."""
        path, off, r = self._locate(name)
        buf = pinned_empty(r["nbytes"])
        self.bytes_read += read_ranges(path, [(off, r["nbytes"], buf.data_ptr())], self.threads)
        return self._view(buf, r), r["dtype"]

    def tensor(self, name: str, device="cuda", staging: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A whole tensor straight into HBM (pread through a pinned double buffer)."""
        path, off, r = self._locate(name)
        out = torch.empty(r["nbytes"], dtype=torch.uint8, device=device)
        st = staging if staging is not None else pinned_empty(min(r["nbytes"], 64 << 20) + 8192)
        read_to_device(path, [(off, r["nbytes"], out.data_ptr())], st, threads=self.threads)
        self.bytes_read += r["nbytes"]
        return self._view(out, r)

    def rows(self, name: str, indices) -> torch.Tensor:
        """The given rows of a 2-D tensor (``loader.py:163-180``: 14 KiB per embedding row
        instead of the whole table), one range per row, read together."""
        path, off, r = self._locate(name)
        cols = r["shape"][1]
        stride = cols * DTYPE_BYTES[r["dtype"]]
        idx = [int(i) for i in indices]
        buf = pinned_empty(stride * len(idx))
        self.bytes_read += read_ranges(path, [(off + i * stride, stride, buf.data_ptr() + j * stride)
                                              for j, i in enumerate(idx)], self.threads)
        return self._view(buf, r, [len(idx), cols])

    def row_block(self, name: str, start: int, n: int) -> torch.Tensor:
        """Rows [start, start + n) of a 2-D tensor (``loader.py:182-193``, the lm_head
        stream)."""
        path, off, r = self._locate(name)
        cols = r["shape"][1]
        stride = cols * DTYPE_BYTES[r["dtype"]]
        buf = pinned_empty(stride * n)
        self.bytes_read += read_ranges(path, [(off + start * stride, stride * n, buf.data_ptr())], self.threads)
        return self._view(buf, r, [n, cols])

    def expert_names(self, layer: int, expert, which: str) -> tuple[str, str]:
        part = "shared_expert" if expert == "shared" else f"experts.{int(expert)}"
        base = f"language_model.model.layers.{layer}.block_sparse_moe.{part}.{which}"
        return base + ".weight_packed", base + ".weight_scale"

    def expert_source(self, layer: int, expert, which: str) -> tuple[torch.Tensor, torch.Tensor]:
        """One MXFP4 projection as (packed u8 [N, K/2], scales u8 [N, K/32]) in pinned host
        memory (``loader.py:229-266``): one read when the scale tensor follows the packed
        one in the same shard, two otherwise; scale bytes must lie in 2..252
        (``mxfp4.py:58-65``)."""
        na, nb = self.expert_names(layer, expert, which)
        pa, oa, ra = self._locate(na)
        pb, ob, rb = self._locate(nb)
        buf = pinned_empty(ra["nbytes"] + rb["nbytes"])
        if pa == pb and oa + ra["nbytes"] == ob:
            got = read_ranges(pa, [(oa, ra["nbytes"] + rb["nbytes"], buf.data_ptr())], self.threads)
        else:
            got = read_ranges(pa, [(oa, ra["nbytes"], buf.data_ptr())], self.threads)
            got += read_ranges(pb, [(ob, rb["nbytes"], buf.data_ptr() + ra["nbytes"])], self.threads)
        packed = buf[:ra["nbytes"]].view(ra["shape"][0], ra["shape"][1])
        scales = buf[ra["nbytes"]:].view(rb["shape"][0], rb["shape"][1])
        lo, hi = int(scales.min()), int(scales.max())
        if lo < 2 or hi > 252:
            raise ValueError(f"Unsupported MXFP4 scale range {lo}..{hi}; require 2..252 "
                             "to avoid Metal subnormal flushing, overflow, and E8M0 NaN")
        self.bytes_read += got
        self.expert_bytes += got
        self.experts_loaded += 1
        return packed, scales

    def moe_weights(self, layer: int, device="cuda") -> dict:
        """The dense weights ``LatentMoE`` takes as ``w`` (``loader.py:30-33,281-282``),
        in HBM, for the keys the layer has."""
        p = f"language_model.model.layers.{layer}.block_sparse_moe."
        st = None
        out = {}
        for k in MOE_KEYS:
            if p + k not in self.recs:
                continue
            if st is None:
                st = pinned_empty(64 << 20)
            out[k] = self.tensor(p + k, device=device, staging=st)
        return out


__all__ = ["classify", "read_header", "manifest_records", "build_manifest", "load_manifest", "read_ranges",
           "read_to_device", "TensorSource", "MOE_KEYS"]
