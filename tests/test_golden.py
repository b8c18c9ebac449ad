"""Pins the oracle and the library's host-side reader to the reference's own
test expectations (CPU only).

Reference tests restated here:
  crates/vocal-model/src/retrieval.rs:291-338   parser byte tests
  crates/vocal-cpu/src/retrieval.rs:87-97        AVX2 unaligned-tail distance
  crates/vocal-directml/src/runtime.rs:592-628   checked-in IVF fixtures
  crates/vocal-tensorrt/src/retrieval/tests.rs:8-13  buffer-capacity checks
"""
import os
import sys
import struct

import numpy as np
import pytest

from conftest import golden


# ---------------------------------------------------------------- parser tests
def _parsers(oracle):
    from vfr import RetrievalIndex

    def oracle_parse(b):
        ix = oracle.OracleIndex.from_faiss(b)
        return ix.vectors().ravel(), ix.ids(), ix.offsets(), ix.nprobe

    def native_parse(b):
        ix = RetrievalIndex.from_faiss(b)
        return ix.vectors().ravel(), ix.ids(), ix.offsets(), ix.nprobe()

    return {"oracle": oracle_parse, "native": native_parse}


@pytest.mark.parametrize("impl", ["oracle", "native"])
def test_flat_and_malformed_inputs(oracle, impl):
    """retrieval.rs:291-306."""
    parse = _parsers(oracle)[impl]
    b = golden("parser_flat.bin")
    vectors, ids, offsets, nprobe = parse(b)
    assert vectors.tolist() == [0.0, 1.0, 2.0, 3.0]
    assert ids.tolist() == [0, 1]
    assert offsets.tolist() == [0, 2] and nprobe == 1
    for n in range(len(b)):
        with pytest.raises(Exception):
            parse(b[:n])
    with pytest.raises(Exception):
        parse(b + b"\0")
    nan = bytearray(b)
    nan[45:49] = struct.pack("<f", float("nan"))
    with pytest.raises(Exception, match="non-finite"):
        parse(bytes(nan))


@pytest.mark.parametrize("impl", ["oracle", "native"])
def test_ivf_lists_preserve_vectors_and_ids(oracle, impl):
    """retrieval.rs:307-338."""
    parse = _parsers(oracle)[impl]
    b = golden("parser_ivf.bin")
    vectors, ids, offsets, nprobe = parse(b)
    assert offsets.tolist() == [0, 1, 2]
    assert ids.tolist() == [1, 0]
    assert vectors.tolist() == [4.0, 4.0, 8.0, 8.0]
    assert nprobe == 1
    for n in range(len(b)):
        with pytest.raises(Exception):
            parse(b[:n])
    dup = bytearray(b)
    dup[-8:] = struct.pack("<Q", 1)
    with pytest.raises(Exception, match="unique IDs"):
        parse(bytes(dup))


@pytest.mark.parametrize("impl", ["oracle", "native"])
def test_rejections(oracle, impl):
    """Reader checks (retrieval.rs:83-193, 233-250): metric, trained flag,
    width, list/probe counts, sizes, direct map, trailing bytes."""
    from vfr import faiss_io

    parse = _parsers(oracle)[impl]
    c = np.zeros((2, 3), np.float32)
    v = np.arange(12, dtype=np.float32).reshape(4, 3)
    good = faiss_io.ivf_bytes(c, v, 1, lists=np.array([0, 1, 0, 1]))
    parse(good)
    bad_metric = bytearray(good)
    bad_metric[33:37] = struct.pack("<i", 0)  # inner product
    with pytest.raises(Exception, match="trained L2"):
        parse(bytes(bad_metric))
    untrained = bytearray(good)
    untrained[32] = 0
    with pytest.raises(Exception, match="trained L2"):
        parse(bytes(untrained))
    with pytest.raises(Exception, match="list/probe"):
        parse(faiss_io.ivf_bytes(c, v, 3, lists=np.array([0, 1, 0, 1])))
    with pytest.raises(Exception, match="supported FAISS types"):
        parse(b"IxPQ" + good[4:])
    wide = np.zeros((1, 4097), np.float32)
    with pytest.raises(Exception, match="width <= 4096"):
        parse(faiss_io.flat_bytes(wide))
    # sparse size directory and a direct map of kind 1 are accepted
    sprs = faiss_io.ivf_bytes(np.zeros((5, 3), np.float32), v, 2, lists=np.array([4, 4, 1, 4]), sizes_kind="sprs",
                              direct_map=1)
    vectors, ids, offsets, _ = parse(sprs)
    assert offsets.tolist() == [0, 0, 1, 1, 1, 4]
    assert ids.tolist() == [2, 0, 1, 3]
    assert vectors.reshape(4, 3)[0].tolist() == v[2].tolist()


def test_parsers_agree_on_random_indexes(oracle):
    from vfr import RetrievalIndex, faiss_io

    rng = np.random.default_rng(7)
    for trial in range(6):
        d = int(rng.integers(1, 70))
        n = int(rng.integers(1, 300))
        nlist = int(rng.integers(1, 12))
        c = rng.standard_normal((nlist, d), dtype=np.float32)
        v = rng.standard_normal((n, d), dtype=np.float32)
        b = faiss_io.ivf_bytes(c, v, int(rng.integers(1, nlist + 1)), sizes_kind=["full", "sprs", None][trial % 3])
        a = oracle.OracleIndex.from_faiss(b)
        r = RetrievalIndex.from_faiss(b)
        assert np.array_equal(a.vectors(), r.vectors()) and np.array_equal(a.ids(), r.ids())
        assert np.array_equal(a.offsets(), r.offsets()) and np.array_equal(a.centroids(), r.centroids())
        assert a.nprobe == r.nprobe()


def test_vfrm_package(oracle):
    """RetrievalIndex::from_package (retrieval.rs:45-57) through a VFRM image."""
    from vfr import RetrievalIndex, faiss_io

    idx = golden("ivf-small-probe2.index")
    image = faiss_io.vfrm_bytes([
        ("aux.retrieval.faiss", 1, (len(idx),), idx),
        ("enc_p.emb_phone.weight", 5, (2, 2), np.ones(4, np.float32).tobytes()),
    ])
    off, n = oracle.vfrm_find_faiss(image)
    assert image[off:off + n] == idx
    ix = RetrievalIndex.from_package(image)
    assert ix.nprobe() == 2 and ix.dimensions() == 2 and len(ix) == 6
    assert RetrievalIndex.from_package(image, feature_dims=2) is not None
    with pytest.raises(Exception, match="feature width"):
        RetrievalIndex.from_package(image, feature_dims=768)
    none = faiss_io.vfrm_bytes([("enc_p.emb_phone.weight", 5, (2, 2), np.ones(4, np.float32).tobytes())])
    assert RetrievalIndex.from_package(none) is None and oracle.vfrm_find_faiss(none) is None
    wrong_dtype = faiss_io.vfrm_bytes([("aux.retrieval.faiss", 2, (len(idx) // 4,), idx[: len(idx) // 4 * 4])])
    with pytest.raises(Exception, match="byte tensor"):
        RetrievalIndex.from_package(wrong_dtype)
    with pytest.raises(Exception):
        RetrievalIndex.from_package(b"VFRM\0\0\0\2" + image[8:])


# ---------------------------------------------------------------- distances
def test_vector_distance_handles_unaligned_tail(oracle):
    """crates/vocal-cpu/src/retrieval.rs:87-97, plus: the portable lane-order
    restatement equals the AVX2 intrinsics bit for bit."""
    a = np.arange(771, dtype=np.float32) / np.float32(100.0)
    b = (np.arange(771) % 13).astype(np.float32)
    actual = oracle.l2(a[1:], b[1:], "avx2")
    expected = oracle.l2(a[1:], b[1:], "scalar")
    assert abs(actual - expected) < expected * 1e-5
    rng = np.random.default_rng(3)
    for d in (1, 7, 8, 33, 256, 768, 770, 4096):
        x, y = rng.standard_normal((2, d), dtype=np.float32)
        assert oracle.l2(x, y, "avx2") == oracle.l2(x, y, "lanes")


# ---------------------------------------------------------------- DML fixtures
QUERIES = np.array([[0, 1], [10, 1.2], [21, 0], [30, 1.5]], np.float32)


def test_dml_fixture_expectations_on_oracle(oracle):
    """crates/vocal-directml/src/runtime.rs:596-625 with ratio 1.  The CPU
    reference returns `IVF search selected no candidate` for frame 2 at
    nprobe=1 (nearest list empty); the CUDA reference keeps the query."""
    for name, nprobe in [("ivf-small-probe1.index", 1), ("ivf-small-probe2.index", 2)]:
        ix = oracle.OracleIndex.from_faiss(golden(name))
        assert ix.nprobe == nprobe and ix.offsets().tolist() == [0, 2, 4, 4, 6]
        out, status = ix.blend(QUERIES, 1.0)
        # exact match: the CPU path weights it 1/(1e-12)^2 in f64 rather than
        # one-hot (DirectML/CUDA), so other probed rows leak in below 1e-20
        assert np.abs(out[0] - [0.0, 1.0]).max() < 1e-20
        if nprobe == 1:
            assert status.tolist() == [0, 0, 2, 0]
            assert out[2].tolist() == [21.0, 0.0]  # untouched row
        else:
            assert status.tolist() == [0, 0, 0, 0]
            assert abs(out[2, 0] - 30.0) < 2e-5


# SHA-256 of the reference's checked-in DirectML fixtures
# (crates/vocal-directml/tests/fixtures/ivf-small-probe{1,2}.index, 299 bytes
# each); the committed golden files must hash to the same values.
REFERENCE_FIXTURE_SHA256 = {
    "ivf-small-probe1.index": "d700e66c191c80bc75ab7a22d9e0e31d145eec90e0af1f56f0b9f0e3314cacbd",
    "ivf-small-probe2.index": "c7ffa837f091abf7e56a4f84b68bf1ee282adb4241ec3732276a9dc632bab550",
}


def test_reference_fixture_bytes():
    """The committed fixtures equal the reference's checked-in files (by
    SHA-256), and this repository's FAISS writer regenerates them."""
    import hashlib

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    import make_golden

    for name, digest in REFERENCE_FIXTURE_SHA256.items():
        data = golden(name)
        assert len(data) == 299
        assert hashlib.sha256(data).hexdigest() == digest
        assert make_golden.FIXTURES[name]() == data


# ---------------------------------------------------------------- boundary checks
def test_rejects_undersized_or_overflowing_bindings():
    """crates/vocal-tensorrt/src/retrieval/tests.rs:8-13."""
    from vfr import validate_blend_buffers

    validate_blend_buffers(140, 768, 140 * 768 * 4, 4)
    with pytest.raises(ValueError):
        validate_blend_buffers(140, 768, 140 * 768 * 4 - 1, 4)
    with pytest.raises(ValueError):
        validate_blend_buffers(140, 768, 140 * 768 * 4, 3)
    with pytest.raises(ValueError):
        validate_blend_buffers(2**64 - 1, 768, 2**64 - 1, 4)
