// Host-side loader: the bounded FAISS reader and the VFRM tensor lookup.
//
// Restates RetrievalIndex::from_faiss (crates/vocal-model/src/retrieval.rs:
// 62-193) with its Reader helpers (:200-268): only little-endian FAISS
// IndexFlatL2 ("IxF2") and IndexIVFFlat ("IwFl") with L2 metric, a Flat-L2
// coarse quantizer and ArrayInvertedLists are accepted; every size is checked
// before allocation, non-finite floats and trailing bytes are rejected, and
// IVF ids must be a permutation of 0..ntotal.  A Flat index becomes one list
// with a zero centroid and nprobe 1.  Error messages keep the reference's
// wording so callers see the same diagnostics.
#include <algorithm>
#include <cmath>
#include <limits>

#include "vfr_common.h"

namespace vfr {
namespace {

[[noreturn]] void bad(const char *message) {
    throw std::runtime_error(std::string("RVC retrieval index: ") + message);
}

class ByteReader {
public:
    ByteReader(const uint8_t *bytes, size_t length) : bytes_(bytes), length_(length) {}

    size_t remaining() const { return length_ - position_; }

    const uint8_t *take(size_t count) {
        if (count > length_ - position_) bad("truncated index");
        const uint8_t *p = bytes_ + position_;
        position_ += count;
        return p;
    }
    uint32_t tag() {
        const uint8_t *p = take(4);
        uint32_t v;
        std::memcpy(&v, p, 4);
        return v;
    }
    uint64_t u64() {
        const uint8_t *p = take(8);
        uint64_t v = 0;
        for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
        if (v > std::numeric_limits<size_t>::max()) bad("size overflow");
        return v;
    }
    void skip_elements(uint64_t count, uint64_t size) {
        if (size != 0 && count > std::numeric_limits<size_t>::max() / size) bad("size overflow");
        take(static_cast<size_t>(count * size));
    }
    // FAISS index header: d:i32, ntotal:i64, 16 legacy bytes, is_trained:u8, metric:i32.
    void header(uint64_t &d, uint64_t &count) {
        int32_t dim = static_cast<int32_t>(tag());
        uint64_t n = u64();
        take(16);
        uint8_t trained = take(1)[0];
        int32_t metric = static_cast<int32_t>(tag());
        if (dim < 1 || dim > 4096 || n == 0 || n > static_cast<uint64_t>(INT32_MAX) || trained != 1 || metric != 1)
            bad("requires a populated, trained L2 index, width <= 4096 and i32 row count");
        d = static_cast<uint64_t>(dim);
        count = n;
    }
    // `count` little-endian f32 values (after an optional u64 length prefix),
    // appended to `out`; all must be finite.
    void floats(uint64_t count, bool length_prefix, std::vector<float> &out) {
        if (length_prefix && u64() != count) bad("float vector length mismatch");
        if (count > std::numeric_limits<size_t>::max() / 4) bad("float shape overflow");
        const uint8_t *p = take(static_cast<size_t>(count * 4));
        size_t base = out.size();
        out.resize(base + count);
        std::memcpy(out.data() + base, p, count * 4);
        for (size_t i = base; i < out.size(); ++i)
            if (!std::isfinite(out[i])) bad("non-finite vector");
    }

private:
    const uint8_t *bytes_;
    size_t length_;
    size_t position_ = 0;
};

constexpr uint32_t fourcc(const char (&s)[5]) {
    return uint32_t(uint8_t(s[0])) | uint32_t(uint8_t(s[1])) << 8 | uint32_t(uint8_t(s[2])) << 16 |
           uint32_t(uint8_t(s[3])) << 24;
}

uint64_t le64(const uint8_t *p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
    return v;
}

}  // namespace

// The structure walk: every check of RetrievalIndex::from_faiss that does
// not depend on the row payload runs here, in the reference's order, and
// throws at once.  The payload checks (finite rows, unique ids) are left to
// the caller, which reports the fault that comes first in the file
// (first_fault), so a host parse and a device ingest raise the same error.
FaissLayout faiss_layout(const uint8_t *bytes, size_t length) {
    require(bytes != nullptr || length == 0, "null FAISS byte buffer");
    ByteReader r(bytes, length);
    FaissLayout L;
    uint32_t kind = r.tag();
    uint64_t d = 0, count = 0;
    r.header(d, count);
    if (kind == fourcc("IxF2")) {
        if (count > std::numeric_limits<uint64_t>::max() / d) bad("shape overflow");
        if (r.u64() != d * count) bad("float vector length mismatch");
        if (d * count > std::numeric_limits<size_t>::max() / 4) bad("float shape overflow");
        const size_t pos = static_cast<size_t>(r.take(static_cast<size_t>(d * count * 4)) - bytes);
        L.lists.push_back({pos, FaissLayout::kImplicitIds, count});
        L.centroids.assign(d, 0.f);
        L.offsets = {0, static_cast<int32_t>(count)};
        L.nprobe = 1;
        L.nlist = 1;
        // checked after the rows, like the reference's final trailing check
        L.trailing = r.remaining() != 0;
    } else if (kind == fourcc("IwFl")) {
        uint64_t nlist = r.u64();
        uint64_t nprobe = r.u64();
        if (nlist == 0 || nprobe == 0 || nprobe > nlist || nlist > length / 8) bad("invalid IVF list/probe count");
        if (r.tag() != fourcc("IxF2")) bad("IVF requires a Flat-L2 coarse quantizer");
        uint64_t cd = 0, cc = 0;
        r.header(cd, cc);
        if (cd != d || cc != nlist) bad("coarse quantizer shape mismatch");
        if (nlist > std::numeric_limits<uint64_t>::max() / d) bad("centroid shape overflow");
        r.floats(nlist * d, true, L.centroids);
        // Direct maps only accelerate id lookups; they carry no search data.
        uint8_t map_kind = r.take(1)[0];
        uint64_t map_len = r.u64();
        if (map_kind > 2 || (map_kind == 0 && map_len != 0) || (map_kind == 1 && map_len != count))
            bad("invalid direct map");
        r.skip_elements(map_len, 8);
        if (map_kind == 2) r.skip_elements(r.u64(), 16);
        if (r.tag() != fourcc("ilar")) bad("only ArrayInvertedLists is supported");
        if (r.u64() != nlist || r.u64() != d * 4) bad("inverted-list layout mismatch");
        uint32_t sizes_kind = r.tag();
        uint64_t sizes_len = r.u64();
        std::vector<uint64_t> sizes(nlist, 0);  // nlist <= length / 8 bounds this
        if (sizes_kind == fourcc("full") && sizes_len == nlist) {
            for (auto &s : sizes) s = r.u64();
        } else if (sizes_kind == fourcc("sprs") && sizes_len % 2 == 0 && sizes_len / 2 <= nlist) {
            for (uint64_t e = 0; e < sizes_len / 2; ++e) {
                uint64_t list = r.u64();
                uint64_t size = r.u64();
                if (list >= nlist || size == 0 || sizes[list] != 0) bad("invalid sparse list directory");
                sizes[list] = size;
            }
        } else {
            bad("invalid inverted-list size directory");
        }
        uint64_t total = 0;
        for (uint64_t s : sizes) {
            if (s > std::numeric_limits<uint64_t>::max() - total) bad("list size overflow");
            total += s;
        }
        if (total != count) bad("list sizes disagree with ntotal");
        if (count > std::numeric_limits<uint64_t>::max() / (d * 4 + 8)) bad("payload overflow");
        if (count * (d * 4 + 8) != r.remaining()) bad("truncated or trailing IVF payload");
        L.lists.reserve(nlist);
        L.offsets.reserve(nlist + 1);
        L.offsets.push_back(0);
        for (uint64_t s : sizes) {
            const size_t vec_pos = static_cast<size_t>(r.take(static_cast<size_t>(s * d * 4)) - bytes);
            const size_t id_pos = static_cast<size_t>(r.take(static_cast<size_t>(s * 8)) - bytes);
            L.lists.push_back({vec_pos, id_pos, s});
            L.offsets.push_back(L.offsets.back() + static_cast<int32_t>(s));
        }
        L.nprobe = static_cast<int32_t>(nprobe);
        L.nlist = static_cast<int32_t>(nlist);
    } else {
        bad("supported FAISS types are IxF2 and IwFl (L2 Flat/IVFFlat)");
    }
    L.d = static_cast<int32_t>(d);
    L.n = static_cast<int64_t>(count);
    return L;
}

size_t FaissLayout::row_position(uint64_t element) const {
    const uint64_t row = element / static_cast<uint64_t>(d);
    // the list holding `row`: offsets is non-decreasing, lists are in file order
    const auto it = std::upper_bound(offsets.begin(), offsets.end(), static_cast<int32_t>(row));
    const size_t list = static_cast<size_t>(it - offsets.begin()) - 1;
    const uint64_t first = static_cast<uint64_t>(offsets[list]) * static_cast<uint64_t>(d);
    return lists[list].vec_pos + static_cast<size_t>(element - first) * 4;
}

size_t scan_ids(const FaissLayout &L, const uint8_t *bytes, std::vector<int32_t> &ids) {
    ids.resize(static_cast<size_t>(L.n));
    if (L.lists.size() == 1 && L.lists[0].id_pos == FaissLayout::kImplicitIds) {
        for (int64_t i = 0; i < L.n; ++i) ids[i] = static_cast<int32_t>(i);
        return FaissLayout::kNoFault;
    }
    std::vector<uint8_t> seen(static_cast<size_t>(L.n), 0);
    size_t row = 0;
    for (const auto &list : L.lists) {
        const uint8_t *p = bytes + list.id_pos;
        for (uint64_t i = 0; i < list.size; ++i, ++row) {
            const uint64_t id = le64(p + 8 * i);
            if (id >= static_cast<uint64_t>(L.n) || seen[id]) return list.id_pos + 8 * i;
            seen[id] = 1;
            ids[row] = static_cast<int32_t>(id);
        }
    }
    return FaissLayout::kNoFault;
}

void raise_first_fault(const FaissLayout &L, size_t nonfinite_pos, size_t bad_id_pos) {
    if (nonfinite_pos != FaissLayout::kNoFault || bad_id_pos != FaissLayout::kNoFault) {
        if (nonfinite_pos < bad_id_pos) bad("non-finite vector");
        bad("RVC requires unique IDs in 0..ntotal");
    }
    if (L.trailing) bad("unexpected trailing data");
}

HostIndex parse_faiss(const uint8_t *bytes, size_t length) {
    FaissLayout L = faiss_layout(bytes, length);
    HostIndex ix;
    ix.vectors.resize(static_cast<size_t>(L.n) * L.d);
    size_t nonfinite = FaissLayout::kNoFault;
    size_t at = 0;
    for (const auto &list : L.lists) {
        const size_t count = static_cast<size_t>(list.size) * L.d;
        float *dst = ix.vectors.data() + at;
        std::memcpy(dst, bytes + list.vec_pos, count * 4);
        if (nonfinite == FaissLayout::kNoFault)
            for (size_t i = 0; i < count; ++i)
                if (!std::isfinite(dst[i])) {
                    nonfinite = list.vec_pos + i * 4;
                    break;
                }
        at += count;
    }
    const size_t bad_id = scan_ids(L, bytes, ix.ids);
    raise_first_fault(L, nonfinite, bad_id);
    ix.d = L.d;
    ix.nlist = L.nlist;
    ix.nprobe = L.nprobe;
    ix.n = L.n;
    ix.centroids = std::move(L.centroids);
    ix.offsets = std::move(L.offsets);
    return ix;
}

// Directory walk of a VFRM v1 image (crates/vocal-model/src/inspection.rs:
// 70-178): 64-byte header (magic "VFRM\0\0\0\1", flags, header size, config
// length, tensor count, directory length, data offset), JSON config, then
// entries name_len:u32, dtype:u8, rank:u8, reserved:u16, name, shape:u64[rank],
// offset:u64, length:u64.  Returns whether aux.retrieval.faiss is present; its
// dtype must be U8 with shape [length] (retrieval.rs:49-51).
bool find_vfrm_faiss(const uint8_t *b, size_t len, size_t *offset, size_t *size) {
    static const uint8_t magic[8] = {'V', 'F', 'R', 'M', 0, 0, 0, 1};
    auto invalid = [](const char *what) {
        throw std::runtime_error(std::string("invalid VFRM cache: ") + what);
    };
    if (len < 64 || std::memcmp(b, magic, 8) != 0) invalid("bad magic/version");
    uint32_t header_size;
    std::memcpy(&header_size, b + 12, 4);
    uint64_t meta_len = le64(b + 16), count = le64(b + 24), dir_len = le64(b + 32), data_off = le64(b + 40);
    if (header_size != 64 || meta_len > len || dir_len > len || count > 100000) invalid("invalid header bounds");
    uint64_t dir_off = 64 + meta_len;
    if (dir_off + dir_len > len || data_off < dir_off + dir_len || data_off > len) invalid("invalid header bounds");
    const uint8_t *dp = b + dir_off;
    uint64_t pos = 0;
    bool found = false;
    static const uint64_t element_size[7] = {0, 1, 4, 8, 2, 4, 2};  // package.rs:54-66 codes 1..6
    for (uint64_t t = 0; t < count; ++t) {
        if (pos + 8 > dir_len) invalid("tensor directory length mismatch");
        uint32_t name_len;
        std::memcpy(&name_len, dp + pos, 4);
        uint8_t dtype = dp[pos + 4], rank = dp[pos + 5];
        pos += 8;
        if (dtype < 1 || dtype > 6) invalid("unknown tensor dtype");
        if (name_len == 0 || name_len > 65535 || rank > 64) invalid("invalid tensor directory entry");
        if (pos + name_len + 8ull * rank + 16 > dir_len) invalid("tensor directory length mismatch");
        const uint8_t *name = dp + pos;
        pos += name_len;
        uint64_t expected = element_size[dtype], dim0 = 0;
        for (uint32_t k = 0; k < rank; ++k) {
            uint64_t dim = le64(dp + pos + 8ull * k);
            if (k == 0) dim0 = dim;
            if (dim != 0 && expected > std::numeric_limits<uint64_t>::max() / dim) invalid("shape overflow");
            expected *= dim;
        }
        pos += 8ull * rank;
        uint64_t toff = le64(dp + pos), tlen = le64(dp + pos + 8);
        pos += 16;
        if (expected != tlen || toff < data_off || toff > len || tlen > len - toff)
            invalid("invalid tensor shape or data range");
        if (name_len == 19 && std::memcmp(name, "aux.retrieval.faiss", 19) == 0) {
            if (dtype != 1 || rank != 1 || dim0 != tlen) bad("expected a byte tensor for aux.retrieval.faiss");
            *offset = static_cast<size_t>(toff);
            *size = static_cast<size_t>(tlen);
            found = true;
        }
    }
    if (pos != dir_len) invalid("tensor directory length mismatch");
    return found;
}

}  // namespace vfr
