"""Regenerates the committed golden fixtures in this directory.

Everything here is rebuilt with this repository's own FAISS byte writer
(vocal-fast-rs_b200/vfr/faiss_io.py) from values published in the reference's
tests, so the fixtures pin the reader and the search semantics without FAISS:

* parser_flat.bin / parser_ivf.bin -- the byte strings that the reference unit
  tests build by hand (crates/vocal-model/src/retrieval.rs:274-338):
  Flat d=2 n=2 values [0,1,2,3]; IVF nlist=2 nprobe=1 with lists
  [(4,4) id 1], [(8,8) id 0].
* ivf-small-probe1.index / ivf-small-probe2.index -- the DirectML retrieval
  fixtures (crates/vocal-directml/tests/fixtures/README.md): centroids
  (0,0),(10,0),(20,0),(30,0); vectors (0,1),(0,2),(10,1),(10,2),(30,1),(30,2)
  added in that order; persisted nprobe 1 and 2.  tests/test_golden.py checks
  that they hash (SHA-256) to the reference's checked-in files.

Run: python tests/golden/make_golden.py
"""
import os
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "vocal-fast-rs_b200"))

import numpy as np  # noqa: E402

from vfr import faiss_io  # noqa: E402


def parser_flat() -> bytes:
    return faiss_io.flat_bytes(np.array([[0.0, 1.0], [2.0, 3.0]], np.float32))


def parser_ivf() -> bytes:
    # header(IwFl, d=2, n=2), nlist=2, nprobe=1, the flat() quantizer bytes,
    # no direct map, ilar/full sizes [1,1], lists (4,4)->id 1 and (8,8)->id 0
    flat = parser_flat()
    out = bytearray(b"IwFl" + struct.pack("<iqqqBi", 2, 2, 1 << 20, 1 << 20, 1, 1))
    out += struct.pack("<QQ", 2, 1) + flat
    out += struct.pack("<BQ", 0, 0) + b"ilar" + struct.pack("<QQ", 2, 8)
    out += b"full" + struct.pack("<QQQ", 2, 1, 1)
    for v, label in [(4.0, 1), (8.0, 0)]:
        out += struct.pack("<ffQ", v, v, label)
    return bytes(out)


def dml_fixture(nprobe: int) -> bytes:
    centroids = np.array([[0, 0], [10, 0], [20, 0], [30, 0]], np.float32)
    vectors = np.array([[0, 1], [0, 2], [10, 1], [10, 2], [30, 1], [30, 2]], np.float32)
    return faiss_io.ivf_bytes(centroids, vectors, nprobe)


FIXTURES = {
    "parser_flat.bin": parser_flat,
    "parser_ivf.bin": parser_ivf,
    "ivf-small-probe1.index": lambda: dml_fixture(1),
    "ivf-small-probe2.index": lambda: dml_fixture(2),
}


def main():
    for name, fn in FIXTURES.items():
        with open(os.path.join(HERE, name), "wb") as f:
            f.write(fn())
        print(name, os.path.getsize(os.path.join(HERE, name)))


if __name__ == "__main__":
    main()
