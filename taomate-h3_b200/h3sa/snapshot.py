"""On-disk snapshot of a CleanAVKVCache, for resuming a stream in another request or process.

The reference keeps its clean AV history in process memory only and drops it when a request
ends (``release_retained_state``, T/streaming/runtime.py:439-449); a restart recomputes the
sink. A snapshot stores what the cache needs to continue exactly where it stopped:

* the bookkeeping: committed block serial, per-commit row counts and token tags, the
  contract (local heads, head dim, dtype), layer names, the segmented-FP8 flag;
* per layer, the committed K/V rows in logical order (bf16, ``[rows, heads, head_dim]``);
* for a segmented FP8 cache, each part's e4m3 rows, its per-head K/V scales and its key
  summary, so the restored parts are the same bytes (not a re-quantisation).

File layout (little endian)::

    b"H3SAKVC1" | u64 header bytes | header (JSON, utf-8) | zero padding to 4096
    sections, each starting on a 4096-byte boundary, as listed in the header:
        {"name", "offset", "nbytes", "crc32", "dtype", "shape"}

The rows leave the device through one gather per layer (``kv_copy_rows`` from the pages into
a dense buffer) and come back the same way; pages are not stored, so a restored cache owns a
compact page sequence. Every section carries a CRC-32 that the loader checks before anything
reaches the device.
"""

from __future__ import annotations

import json
import os
import struct
import zlib
from pathlib import Path

import torch

from .cache import CleanAVKVCache, KVContract
from .kernels import kv_copy_rows

MAGIC = b"H3SAKVC1"
FORMAT_VERSION = 1
ALIGN = 4096
_DTYPES = {"bfloat16": torch.bfloat16, "float8_e4m3fn": torch.float8_e4m3fn,
           "float32": torch.float32}


def _dtype_name(dtype: torch.dtype) -> str:
    for name, d in _DTYPES.items():
        if d == dtype:
            return name
    raise ValueError(f"snapshot cannot store dtype {dtype}")


def _host_bytes(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()


class _Writer:
    def __init__(self) -> None:
        self.sections: list[dict] = []
        self.blobs: list[bytes] = []
        self.cursor = 0

    def add(self, name: str, t: torch.Tensor) -> None:
        data = _host_bytes(t)
        self.sections.append({"name": name, "offset": self.cursor, "nbytes": len(data),
                              "crc32": zlib.crc32(data), "dtype": _dtype_name(t.dtype),
                              "shape": [int(s) for s in t.shape]})
        self.blobs.append(data)
        self.cursor += (len(data) + ALIGN - 1) // ALIGN * ALIGN


def save_cache(cache: CleanAVKVCache, path: str | os.PathLike) -> None:
    """Write ``cache`` to ``path`` (replaced atomically: a temporary file is renamed)."""

    cache._require_valid()
    if cache.clean_commit_active:
        raise RuntimeError("cannot snapshot the H3 cache during a clean commit")
    w = _Writer()
    layers = {}
    for name in cache.layer_names:
        paged = cache._layers.get(name)
        if paged is None or paged.history_rows == 0:
            continue
        key, value = paged.materialize(paged.history_rows)
        w.add(f"{name}/key", key)
        w.add(f"{name}/value", value)
        entry = {"rows": paged.history_rows}
        seg = paged.fp8
        if seg is not None and seg.starts:
            total = sum(seg.rows)
            k8 = torch.empty(total, seg.heads, cache.contract.head_dim, dtype=torch.float8_e4m3fn,
                             device=seg.store.device)
            v8 = torch.empty_like(k8)
            cursor = 0
            for s0, n in zip(seg.starts, seg.rows):
                kv_copy_rows([seg.store.key, seg.store.value], [k8, v8], count=n,
                             src_table=seg.store.table, src_start=s0, dst_start=cursor)
                cursor += n
            w.add(f"{name}/fp8_key", k8)
            w.add(f"{name}/fp8_value", v8)
            w.add(f"{name}/k_scale", seg.k_scale)
            w.add(f"{name}/v_scale", seg.v_scale)
            w.add(f"{name}/key_summary", seg.key_summary)
            entry["parts"] = list(seg.rows)
        layers[name] = entry
    c = cache.contract
    header = {
        "format": FORMAT_VERSION,
        "contract": {"local_heads": c.local_heads, "head_dim": c.head_dim,
                     "dtype": _dtype_name(c.dtype), "device_type": c.device_type},
        "layer_names": list(cache.layer_names),
        "segmented_fp8_history": bool(cache.segmented_fp8_history),
        "block_index": cache._block_index,
        "commit_token_counts": list(cache._commit_token_counts),
        "commit_token_tags": [list(t) for t in cache._commit_token_tags],
        "layers": layers,
        "sections": w.sections,
    }
    head = json.dumps(header, separators=(",", ":")).encode()
    base = (len(MAGIC) + 8 + len(head) + ALIGN - 1) // ALIGN * ALIGN
    path = Path(path)
    tmp = path.with_name(path.name + ".tmp")
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        f.write(b"\0" * (base - len(MAGIC) - 8 - len(head)))
        for sec, blob in zip(w.sections, w.blobs):
            f.seek(base + sec["offset"])
            f.write(blob)
        f.truncate(base + w.cursor)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def read_header(path: str | os.PathLike) -> tuple[dict, int]:
    """The snapshot's header and the file offset of its first section (no device work)."""

    with open(path, "rb") as f:
        magic = f.read(len(MAGIC))
        if magic != MAGIC:
            raise ValueError(f"{path}: not an H3 cache snapshot")
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: truncated snapshot header")
        (n,) = struct.unpack("<Q", raw)
        head = f.read(n)
        if len(head) != n:
            raise ValueError(f"{path}: truncated snapshot header")
    header = json.loads(head.decode())
    if header.get("format") != FORMAT_VERSION:
        raise ValueError(f"{path}: snapshot format {header.get('format')} is not "
                         f"{FORMAT_VERSION}")
    base = (len(MAGIC) + 8 + n + ALIGN - 1) // ALIGN * ALIGN
    return header, base


def load_cache(path: str | os.PathLike, *, device: torch.device | str | None = None,
               contract: KVContract | None = None,
               initial_pages: int = 8) -> CleanAVKVCache:
    """Rebuild the cache a snapshot holds on ``device``. A given ``contract`` must match the
    stored one (a resumed model must shard its heads the same way)."""

    header, base = read_header(path)
    c = header["contract"]
    stored = KVContract(local_heads=int(c["local_heads"]), head_dim=int(c["head_dim"]),
                        dtype=_DTYPES[c["dtype"]], device_type=c["device_type"])
    if contract is not None and contract != stored:
        raise ValueError(f"snapshot contract {stored} differs from {contract}")
    sections = {s["name"]: s for s in header["sections"]}
    size = os.path.getsize(path)
    blobs: dict[str, torch.Tensor] = {}
    with open(path, "rb") as f:
        for name, s in sections.items():
            if base + s["offset"] + s["nbytes"] > size:
                raise ValueError(f"{path}: section {name} is truncated")
            f.seek(base + s["offset"])
            data = f.read(s["nbytes"])
            if zlib.crc32(data) != s["crc32"]:
                raise ValueError(f"{path}: section {name} fails its CRC-32 check")
            t = torch.frombuffer(bytearray(data), dtype=torch.uint8)
            blobs[name] = t.view(_DTYPES[s["dtype"]]).reshape(s["shape"])
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    cache = CleanAVKVCache(stored, layer_names=tuple(header["layer_names"]), device=dev,
                           initial_pages=initial_pages,
                           segmented_fp8_history=bool(header["segmented_fp8_history"]))
    for name, entry in header["layers"].items():
        rows = int(entry["rows"])
        paged = cache.layer(name, dev)
        key = blobs[f"{name}/key"].pin_memory().to(dev, non_blocking=True)
        value = blobs[f"{name}/value"].pin_memory().to(dev, non_blocking=True)
        if tuple(key.shape) != (rows, stored.local_heads, stored.head_dim):
            raise ValueError(f"{path}: {name} key rows do not match the header")
        paged.write(key, value, start=0, count=rows)
        paged.history_rows = rows
        parts = entry.get("parts")
        if parts:
            seg = paged.fp8
            k8 = blobs[f"{name}/fp8_key"].pin_memory().to(dev, non_blocking=True)
            v8 = blobs[f"{name}/fp8_value"].pin_memory().to(dev, non_blocking=True)
            cursor = 0
            for n in parts:
                s0 = seg.end
                seg.store.reserve(s0 + n)
                kv_copy_rows([k8, v8], [seg.store.key, seg.store.value], count=n,
                             src_start=cursor, dst_table=seg.store.table, dst_start=s0)
                seg.starts.append(s0)
                seg.rows.append(n)
                cursor += n
            seg.k_scale = blobs[f"{name}/k_scale"].to(dev)
            seg.v_scale = blobs[f"{name}/v_scale"].to(dev)
            seg.key_summary = blobs[f"{name}/key_summary"].to(dev)
    cache._block_index = int(header["block_index"])
    cache._commit_token_counts = [int(n) for n in header["commit_token_counts"]]
    cache._commit_token_tags = [tuple(int(t) for t in tags)
                                for tags in header["commit_token_tags"]]
    if any(sum(cache._commit_token_counts) != int(e["rows"]) for e in header["layers"].values()):
        raise ValueError(f"{path}: layer rows differ from the commit counts")
    return cache


__all__ = ["FORMAT_VERSION", "load_cache", "read_header", "save_cache"]
