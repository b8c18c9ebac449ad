"""Device ingest of FAISS indexes (`vfr_index_load`, `vfr_index_load_vfrm`,
`vfr_index_load_file`): RetrievalIndex::from_faiss + GpuRetrievalIndex::new
in one pass without a host copy of the rows
(crates/vocal-model/src/retrieval.rs:45-193, crates/vocal-tensorrt/src/
retrieval.rs:27-60).

CPU: every structural error, and the payload errors the host decides (a
duplicate id, and a non-finite row before it), carry the parser's message
and precedence, checked against `vfr_index_parse_faiss` on the reference's
parser bytes and their truncations.
GPU: loaded indexes blend bit-identically to parse + upload (golden IVF
fixtures, random IVF with empty and ragged lists, a flat index large enough
for the multi-threaded staged upload); non-finite rows found on the device
rank against trailing bytes and ids by file position; VFRM images and files;
storage shared between handles loaded from the same bytes.
"""
import ctypes
import struct

import numpy as np
import pytest

from conftest import golden


def _parse_error(data: bytes):
    from vfr import lib

    L = lib.load_library()
    out = ctypes.c_void_p()
    try:
        lib.call(L.vfr_index_parse_faiss, data, len(data), ctypes.byref(out))
    except lib.NativeError as e:
        return str(e)
    L.vfr_index_free(out)
    return None


def _load_error(data: bytes):
    from vfr import lib

    L = lib.load_library()
    out = ctypes.c_void_p()
    buf = np.frombuffer(data, np.uint8) if data else np.zeros(0, np.uint8)
    try:
        lib.call(L.vfr_index_load, buf.ctypes.data if buf.size else None, buf.size, None, ctypes.byref(out))
    except lib.NativeError as e:
        return str(e)
    L.vocal_faiss_gpu_destroy(out)
    return None


HOST_DECIDED = ("non-finite", "unique IDs", "trailing data")


def _structural_cases():
    from vfr import faiss_io

    flat = golden("parser_flat.bin")
    ivf = golden("parser_ivf.bin")
    cases = [flat[:n] for n in range(len(flat))] + [ivf[:n] for n in range(len(ivf))]
    c = np.zeros((2, 3), np.float32)
    v = np.arange(12, dtype=np.float32).reshape(4, 3)
    good = faiss_io.ivf_bytes(c, v, 1, lists=np.array([0, 1, 0, 1]))
    metric = bytearray(good)
    metric[33:37] = struct.pack("<i", 0)
    untrained = bytearray(good)
    untrained[32] = 0
    cases += [bytes(metric), bytes(untrained), faiss_io.ivf_bytes(c, v, 3, lists=np.array([0, 1, 0, 1])),
              b"IxPQ" + good[4:], faiss_io.flat_bytes(np.zeros((1, 4097), np.float32)), good + b"\0", b""]
    return cases


def test_loader_structural_errors_match_parser():
    """Errors raised before any device work: same message as the parser."""
    seen = 0
    for data in _structural_cases():
        want = _parse_error(data)
        assert want is not None
        if any(h in want for h in HOST_DECIDED) and "unique IDs" not in want:
            continue  # needs the device row check
        assert _load_error(data) == want, (len(data), want)
        seen += 1
    assert seen > 40


def test_loader_id_faults_rank_by_file_position():
    """A duplicate id is found on the host; a non-finite row before it in the
    file wins, one after it does not (Reader order, retrieval.rs:140-175)."""
    from vfr import faiss_io

    c = np.zeros((3, 2), np.float32)
    v = np.arange(12, dtype=np.float32).reshape(6, 2)
    lists = np.array([0, 0, 1, 1, 2, 2])
    base = faiss_io.ivf_bytes(c, v, 1, lists=lists)
    from vfr import RetrievalIndex

    ix = RetrievalIndex.from_faiss(base)
    assert ix.offsets().tolist() == [0, 2, 4, 6]
    # payload: per list 2 rows x 2 f32 then 2 u64 ids; lists start after the header
    payload = len(base) - 6 * (2 * 4 + 8)
    list_bytes = 2 * 2 * 4 + 2 * 8

    def patched(nan_list=None, dup_list=None):
        b = bytearray(base)
        if nan_list is not None:
            at = payload + nan_list * list_bytes + 4
            b[at:at + 4] = struct.pack("<f", float("inf"))
        if dup_list is not None:
            at = payload + dup_list * list_bytes + 16 + 8
            b[at:at + 8] = b[at - 8:at]
        return bytes(b)

    for nan_list, dup_list in ((0, 1), (1, 1), (2, 1), (None, 0)):
        data = patched(nan_list, dup_list)
        want = _parse_error(data)
        assert want == ("RVC retrieval index: non-finite vector" if nan_list is not None and nan_list <= dup_list
                        else "RVC retrieval index: RVC requires unique IDs in 0..ntotal")
        assert _load_error(data) == want


# ------------------------------------------------------------------- GPU


def _blend(g, q, ratio, torch):
    x = torch.from_numpy(q.copy()).cuda()
    rate = torch.tensor([ratio], device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        g.blend(x, q.shape[0], rate, stream=s)
    s.synchronize()
    return x.cpu().numpy()


def _same_index(a, b, q, ratio, torch):
    da, db = a.diagnostics(), b.diagnostics()
    for k in ("dimensions", "nlist", "nprobe", "vectors", "tensor_cores", "max_row_norm", "max_row_residual"):
        assert da[k] == db[k], k
    assert np.array_equal(_blend(a, q, ratio, torch).view(np.uint32), _blend(b, q, ratio, torch).view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["ivf-small-probe1.index", "ivf-small-probe2.index"])
def test_load_matches_parse_and_upload_on_fixtures(cuda, name):
    from vfr import GpuRetrievalIndex, RetrievalIndex

    data = golden(name)
    host = RetrievalIndex.from_faiss(data)
    up = GpuRetrievalIndex.upload(host)
    ld = GpuRetrievalIndex.load(data)
    rng = np.random.default_rng(3)
    q = rng.standard_normal((37, host.dimensions())).astype(np.float32)
    _same_index(up, ld, q, 0.75, cuda)
    up.close()
    ld.close()


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(64, 60000, 768, 4), (9, 3000, 256, 2), (1, 100000, 768, 1)])
def test_load_matches_from_arrays_staged(cuda, shape):
    """Payloads above the single-copy size go through the threaded staging:
    a 64-list IVF with empty and ragged lists, a small IVF, a 307 MB flat."""
    from vfr import GpuRetrievalIndex, RetrievalIndex, faiss_io

    nlist, n, d, nprobe = shape
    rng = np.random.default_rng(nlist + n)
    c = rng.standard_normal((nlist, d), dtype=np.float32)
    v = rng.standard_normal((n, d), dtype=np.float32)
    if nlist > 1:
        lists = rng.integers(0, nlist - 3, n)  # the last three lists stay empty
        lists[: n // 3] = 5  # one long list
        data = faiss_io.ivf_bytes(c, v, nprobe, lists=lists)
    else:
        data = faiss_io.flat_bytes(v)
    del v
    host = RetrievalIndex.from_faiss(data)
    ref = GpuRetrievalIndex.from_arrays(host.centroids(), host.offsets(), host.vectors(), host.ids(), host.nprobe())
    ld = GpuRetrievalIndex.load(np.frombuffer(data, np.uint8))
    q = host.vectors()[rng.integers(0, n, 64)] + 0.05 * rng.standard_normal((64, d), dtype=np.float32)
    _same_index(ref, ld, q.astype(np.float32), 0.75, cuda)
    ref.close()
    ld.close()


@pytest.mark.gpu
def test_device_row_check_ranks_with_trailing_bytes(cuda):
    from vfr import GpuRetrievalIndex, faiss_io, lib

    rng = np.random.default_rng(5)
    v = rng.standard_normal((40000, 256), dtype=np.float32)
    data = bytearray(faiss_io.flat_bytes(v))
    header = len(data) - v.size * 4
    ok = bytes(data)
    with pytest.raises(lib.NativeError, match="unexpected trailing data"):
        GpuRetrievalIndex.load(ok + b"\0")
    last = header + (v.size - 3) * 4  # near the end: found by the device scan
    data[last:last + 4] = struct.pack("<f", float("nan"))
    for tail in (b"", b"\0\0"):
        with pytest.raises(lib.NativeError, match="non-finite vector"):
            GpuRetrievalIndex.load(bytes(data) + tail)
    g = GpuRetrievalIndex.load(ok)
    assert g.n == 40000 and g.d == 256
    g.close()


@pytest.mark.gpu
def test_device_row_check_in_ivf_lists(cuda):
    from vfr import GpuRetrievalIndex, RetrievalIndex, faiss_io, lib

    rng = np.random.default_rng(6)
    c = rng.standard_normal((8, 64), dtype=np.float32)
    v = rng.standard_normal((5000, 64), dtype=np.float32)
    data = faiss_io.ivf_bytes(c, v, 2)
    host = RetrievalIndex.from_faiss(data)
    # the first row of the last list, found by value in the image
    row = host.vectors()[host.offsets()[7]]
    at = bytes(data).find(row.tobytes())
    assert at > 0
    bad = bytearray(data)
    bad[at + 8:at + 12] = struct.pack("<f", float("-inf"))
    want = _parse_error(bytes(bad))
    assert "non-finite" in want
    with pytest.raises(lib.NativeError) as e:
        GpuRetrievalIndex.load(bytes(bad))
    assert str(e.value) == want
    wide = faiss_io.ivf_bytes(np.zeros((40, 4), np.float32), rng.standard_normal((100, 4), dtype=np.float32), 33)
    with pytest.raises(lib.NativeError, match="invalid FAISS GPU IVF configuration"):
        GpuRetrievalIndex.load(wide)


@pytest.mark.gpu
def test_load_vfrm_and_files(cuda, tmp_path):
    from vfr import GpuRetrievalIndex, RetrievalIndex, faiss_io, lib

    idx = golden("ivf-small-probe2.index")
    image = faiss_io.vfrm_bytes([
        ("aux.retrieval.faiss", 1, (len(idx),), idx),
        ("enc_p.emb_phone.weight", 5, (2, 2), np.ones(4, np.float32).tobytes()),
    ])
    none = faiss_io.vfrm_bytes([("enc_p.emb_phone.weight", 5, (2, 2), np.ones(4, np.float32).tobytes())])
    q = np.random.default_rng(8).standard_normal((11, 2)).astype(np.float32)
    up = GpuRetrievalIndex.upload(RetrievalIndex.from_faiss(idx))
    (tmp_path / "voice.index").write_bytes(idx)
    (tmp_path / "voice.vfrm").write_bytes(image)
    (tmp_path / "none.vfrm").write_bytes(none)
    for source in (image, tmp_path / "voice.index", tmp_path / "voice.vfrm", str(tmp_path / "voice.vfrm")):
        g = GpuRetrievalIndex.load(source, feature_dims=2)
        _same_index(up, g, q, 0.5, cuda)
        g.close()
    assert GpuRetrievalIndex.load(none) is None
    assert GpuRetrievalIndex.load(tmp_path / "none.vfrm") is None
    for source in (image, tmp_path / "voice.vfrm"):
        with pytest.raises(lib.NativeError, match="feature width"):
            GpuRetrievalIndex.load(source, feature_dims=768)
    with pytest.raises(lib.NativeError, match="cannot open retrieval index file"):
        GpuRetrievalIndex.load(tmp_path / "missing.index")
    up.close()


@pytest.mark.gpu
def test_shared_storage(cuda):
    """Handles loaded with share=True from the same bytes share the device
    arrays (diagnostics shared_handles), keep their own workspace, counters
    and label base, and outlive each other; other bytes or the exact engine
    get their own arrays."""
    from vfr import GpuRetrievalIndex, faiss_io, lib

    rng = np.random.default_rng(9)
    c = rng.standard_normal((16, 128), dtype=np.float32)
    v = rng.standard_normal((20000, 128), dtype=np.float32)
    data = faiss_io.ivf_bytes(c, v, 4)
    q = v[:50] + 0.01
    a = GpuRetrievalIndex.load(data, share=True)
    b = GpuRetrievalIndex.load(data, share=True, label_base=1000)
    plain = GpuRetrievalIndex.load(data)
    exact = GpuRetrievalIndex.load(data, share=True, engine=lib.ENGINE_EXACT)
    other = GpuRetrievalIndex.load(faiss_io.ivf_bytes(c, v * 2, 4), share=True)
    assert a.diagnostics()["shared_handles"] == 2 and b.diagnostics()["shared_handles"] == 2
    assert plain.diagnostics()["shared_handles"] == 0
    assert exact.diagnostics()["shared_handles"] == 1 and other.diagnostics()["shared_handles"] == 1
    want = _blend(plain, q, 0.75, cuda)
    assert np.array_equal(_blend(a, q, 0.75, cuda), want)
    s = cuda.cuda.Stream()
    dq = cuda.from_numpy(q).cuda()
    cuda.cuda.synchronize()
    with cuda.cuda.stream(s):
        da, la = a.search(dq, stream=s)
        db, lb = b.search(dq, stream=s)
    s.synchronize()
    assert np.array_equal(da.cpu().numpy(), db.cpu().numpy())
    assert np.array_equal(la.cpu().numpy() + 1000, lb.cpu().numpy())
    a.close()
    assert b.diagnostics()["shared_handles"] == 1
    assert np.array_equal(_blend(b, q, 0.75, cuda), want)
    b.close()
    c2 = GpuRetrievalIndex.load(data, share=True)
    assert c2.diagnostics()["shared_handles"] == 1
    assert np.array_equal(_blend(c2, q, 0.75, cuda), want)
    for g in (c2, plain, exact, other):
        g.close()


# ------------------------------------------------------- host-only checks


def _hash(data) -> tuple:
    from vfr import lib

    buf = np.frombuffer(bytes(data), np.uint8) if len(data) else np.zeros(0, np.uint8)
    out = np.zeros(2, np.uint64)
    lib.call(lib.load_library().vfr_index_content_hash, buf.ctypes.data if buf.size else None, buf.size,
             out.ctypes.data)
    return int(out[0]), int(out[1])


def test_content_hash_keys_bytes():
    """The share key: stable for the same bytes, different for any change
    (every byte flipped in turn on a small image, random flips across 1 MiB
    blocks on a large one), the length included."""
    rng = np.random.default_rng(17)
    small = rng.integers(0, 256, 300, dtype=np.uint8).tobytes()
    base = _hash(small)
    assert _hash(small) == base and _hash(bytearray(small)) == base
    seen = {base}
    for i in range(len(small)):
        b = bytearray(small)
        b[i] ^= 0x01
        seen.add(_hash(b))
    assert len(seen) == len(small) + 1
    assert _hash(small + b"\0") != base and _hash(small[:-1]) != base and _hash(b"") != _hash(b"\0")
    big = rng.integers(0, 256, (5 << 20) + 123, dtype=np.uint8)
    hb = _hash(big)
    assert _hash(big.copy()) == hb
    for pos in rng.integers(0, big.size, 8):
        b = big.copy()
        b[pos] ^= 0x80
        assert _hash(b) != hb


def test_file_loader_errors_without_device(tmp_path):
    """Errors raised before any device work carry the parser's message; a
    missing file names the path."""
    import ctypes

    from vfr import lib

    L = lib.load_library()
    out = ctypes.c_void_p()
    with pytest.raises(lib.NativeError, match="cannot open retrieval index file"):
        lib.call(L.vfr_index_load_file, str(tmp_path / "missing.index").encode(), 0, None, ctypes.byref(out))
    flat = golden("parser_flat.bin")
    (tmp_path / "cut.index").write_bytes(flat[:20])
    with pytest.raises(lib.NativeError) as e:
        lib.call(L.vfr_index_load_file, str(tmp_path / "cut.index").encode(), 0, None, ctypes.byref(out))
    assert str(e.value) == _parse_error(flat[:20])
    (tmp_path / "empty.index").write_bytes(b"")
    with pytest.raises(lib.NativeError, match="truncated index"):
        lib.call(L.vfr_index_load_file, str(tmp_path / "empty.index").encode(), 0, None, ctypes.byref(out))
