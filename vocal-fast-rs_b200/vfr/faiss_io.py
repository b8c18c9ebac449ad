"""Writers for the on-disk formats either side of the retrieval path.

* FAISS `IndexFlatL2` ("IxF2") and `IndexIVFFlat` ("IwFl") bytes, in the
  little-endian layout that the reference's bounded reader accepts
  (crates/vocal-model/src/retrieval.rs:62-193): index header (d:i32, ntotal:i64,
  two legacy i64 fields = 1<<20, is_trained:u8, metric:i32), then for Flat the
  length-prefixed f32 payload; for IVF nlist, nprobe, the Flat-L2 coarse
  quantizer, a direct map, and `ilar` ArrayInvertedLists with a `full` or
  `sprs` size directory followed by each list's codes and i64 ids.
* VFRM v1 containers carrying the index as the U8 tensor
  `aux.retrieval.faiss` (crates/vocal-model/src/lib.rs:586-612 writes the same
  header: magic, flags, header size, config length, tensor count, directory
  length, data offset, two reserved u64).

These are plain byte builders with no FAISS dependency; they let tests and the
benchmark exercise the same load path as a real voice index.
"""
from __future__ import annotations

import json
import struct

import numpy as np

LEGACY_DUMMY = 1 << 20
METRIC_L2 = 1


def _index_header(kind: bytes, d: int, ntotal: int, trained: int = 1, metric: int = METRIC_L2) -> bytes:
    return kind + struct.pack("<iqqqBi", d, ntotal, LEGACY_DUMMY, LEGACY_DUMMY, trained, metric)


def flat_bytes(vectors: np.ndarray) -> bytes:
    """FAISS IndexFlatL2 serialisation of `vectors` [n, d]."""
    v = np.ascontiguousarray(vectors, dtype="<f4")
    n, d = v.shape
    return _index_header(b"IxF2", d, n) + struct.pack("<Q", v.size) + v.tobytes()


def assign_lists(centroids: np.ndarray, vectors: np.ndarray) -> np.ndarray:
    """Nearest-centroid list per vector (ties to the lower list id), the
    assignment `IndexIVFFlat::add` makes with a Flat-L2 quantizer."""
    c = np.asarray(centroids, np.float64)
    out = np.empty(len(vectors), np.int64)
    step = 8192
    cn = (c * c).sum(1)
    for s in range(0, len(vectors), step):
        x = np.asarray(vectors[s:s + step], np.float64)
        dist = cn[None, :] - 2.0 * x @ c.T
        out[s:s + step] = dist.argmin(1)
    return out


def ivf_bytes(centroids: np.ndarray, vectors: np.ndarray, nprobe: int, lists: np.ndarray | None = None,
              ids: np.ndarray | None = None, sizes_kind: str | None = None, direct_map: int = 0) -> bytes:
    """FAISS IndexIVFFlat (L2, Flat quantizer, ArrayInvertedLists) bytes.

    `lists[i]` is the inverted list of `vectors[i]` (default: nearest centroid);
    `ids[i]` its label (default: i).  Within a list, vectors keep their input
    order, as FAISS appends them.  `sizes_kind` forces "full"/"sprs"; by default
    FAISS's rule is used ("full" when more than half the lists are non-empty).
    """
    c = np.ascontiguousarray(centroids, dtype="<f4")
    v = np.ascontiguousarray(vectors, dtype="<f4")
    nlist, d = c.shape
    n = v.shape[0]
    if lists is None:
        lists = assign_lists(c, v)
    lists = np.asarray(lists, np.int64)
    if ids is None:
        ids = np.arange(n, dtype=np.int64)
    ids = np.asarray(ids, np.int64)
    order = np.argsort(lists, kind="stable")
    sizes = np.bincount(lists, minlength=nlist).astype(np.uint64)
    out = bytearray()
    out += _index_header(b"IwFl", d, n)
    out += struct.pack("<QQ", nlist, nprobe)
    out += flat_bytes(c)
    if direct_map == 0:
        out += struct.pack("<BQ", 0, 0)
    elif direct_map == 1:
        dm = np.zeros(n, "<i8")
        out += struct.pack("<BQ", 1, n) + dm.tobytes()
    else:
        raise ValueError("direct_map must be 0 or 1")
    out += b"ilar" + struct.pack("<QQ", nlist, d * 4)
    nonempty = int((sizes > 0).sum())
    if sizes_kind is None:
        sizes_kind = "full" if nonempty > nlist // 2 else "sprs"
    if sizes_kind == "full":
        out += b"full" + struct.pack("<Q", nlist) + sizes.astype("<u8").tobytes()
    else:
        pairs = [(l, int(sizes[l])) for l in range(nlist) if sizes[l]]
        out += b"sprs" + struct.pack("<Q", 2 * len(pairs))
        for l, s in pairs:
            out += struct.pack("<QQ", l, s)
    start = 0
    for l in range(nlist):
        cnt = int(sizes[l])
        sel = order[start:start + cnt]
        start += cnt
        out += v[sel].tobytes()
        out += ids[sel].astype("<i8").tobytes()
    return bytes(out)


def vfrm_bytes(tensors: list[tuple[str, int, tuple[int, ...], bytes]], manifest: dict | None = None) -> bytes:
    """A VFRM v1 image.  `tensors` holds (name, dtype code, shape, raw bytes);
    dtype codes follow crates/vocal-model/src/package.rs:54-66
    (1=u8, 2=i32, 3=i64, 4=f16, 5=f32, 6=bf16).  Tensors are 64-byte aligned."""
    config = json.dumps({"manifest": manifest or {"version": "v2"}, "metadata": {}}).encode()
    directory = bytearray()
    tensors = sorted(tensors, key=lambda t: t[0])
    # offsets are known only after the directory length, which does not depend on them
    dir_len = sum(4 + 4 + len(name.encode()) + 8 * len(shape) + 16 for name, _, shape, _ in tensors)
    align = lambda x: (x + 63) // 64 * 64
    data_offset = align(64 + len(config) + dir_len)
    offsets = []
    cur = data_offset
    for _, _, _, data in tensors:
        cur = align(cur)
        offsets.append(cur)
        cur += len(data)
    for (name, dtype, shape, data), off in zip(tensors, offsets):
        nb = name.encode()
        directory += struct.pack("<IBBH", len(nb), dtype, len(shape), 0) + nb
        directory += b"".join(struct.pack("<Q", s) for s in shape)
        directory += struct.pack("<QQ", off, len(data))
    assert len(directory) == dir_len
    head = b"VFRM\0\0\0\x01" + struct.pack("<IIQQQQQQ", 0, 64, len(config), len(tensors), dir_len, data_offset, 0, 0)
    out = bytearray(head + config + bytes(directory))
    out += b"\0" * (data_offset - len(out))
    for (_, _, _, data), off in zip(tensors, offsets):
        out += b"\0" * (off - len(out))
        out += data
    return bytes(out)


def vfrm_with_index(index_bytes: bytes, manifest: dict | None = None) -> bytes:
    """VFRM image holding `index_bytes` as aux.retrieval.faiss (U8, rank 1)."""
    return vfrm_bytes([("aux.retrieval.faiss", 1, (len(index_bytes),), index_bytes)], manifest)
