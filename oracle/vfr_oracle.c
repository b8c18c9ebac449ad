/*
 * vfr_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference CPU retrieval path of
 * MosRat/vocal-fast-rs, used as the parity checker for the CUDA library and as
 * the timed CPU baseline.  Nothing in the product links or calls this file; only
 * tests/, __graft_entry__.smoke() and bench.py (cpu_baseline / --impl reference)
 * load it.
 *
 * Restated reference code (paths inside the reference project):
 *   - FAISS reader:   crates/vocal-model/src/retrieval.rs:62-268
 *                     (Reader::{take,tag,usize,skip_elements,header,floats})
 *   - VFRM container: crates/vocal-model/src/inspection.rs:70-178 and
 *                     crates/vocal-model/src/retrieval.rs:45-57 (from_package)
 *   - distances:      crates/vocal-cpu/src/retrieval.rs:5-26 (scalar_l2, avx2_l2)
 *   - search + blend: crates/vocal-cpu/src/retrieval.rs:27-83 (blend)
 *   - call site:      crates/vocal-cpu/src/pipeline.rs:292-301 (serial per-frame loop)
 *   - protection:     crates/vocal-tensorrt/native/retrieval_protection.cu:4-16
 *                     (protect_features; GPU-only in the reference)
 *   - RVC frontend:   crates/vocal-tensorrt/native/frontend.cpp:36-75 (append the
 *                     last HuBERT frame, nearest 2x, crop, coarse pitch; a
 *                     TensorRT graph in the reference)
 *   - engine frontend: crates/vocal-engine/src/pipeline.rs:75-96 (linear 2x),
 *                     312-333 (protection), 625-633 (f0_to_coarse)
 *   - IVF training:   the library's deterministic trainer (vfr_kmeans,
 *                     vfr_ivf_assign).  The reference trains offline with
 *                     FAISS IndexIVFFlat::train/add (recipe in
 *                     crates/vocal-directml/tests/fixtures/README.md,
 *                     scripts/benchmark-retrieval.py:56-65; FAISS is not
 *                     vendored); the algorithm is FAISS's Clustering with a
 *                     SplitMix64 generator, exact nearest-centroid assignment
 *                     under avx2_l2's order and 64-bit fixed-point means.
 *
 * Arithmetic order is kept exactly: AVX2 8-lane direct-difference squared L2
 * with separate multiply and add, the eight lanes folded left to right, then
 * the scalar tail; f64 inverse-square weights; f32 blend without contraction.
 * Rust's float `Sum` folds from -0.0, which is reproduced here.  Build with
 * -O2 -mavx2 -ffp-contract=off (see oracle/Makefile); never with -ffast-math.
 */
#define _GNU_SOURCE
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORC_K 8

typedef struct orc_index {
    int64_t d;
    int64_t nprobe;
    int64_t nlist;
    int64_t n;
    float *centroids;  /* nlist * d */
    int32_t *offsets;  /* nlist + 1 */
    float *vectors;    /* n * d, inverted-list order */
    int32_t *ids;      /* n, FAISS labels (a permutation of 0..n) */
} orc_index;

/* ------------------------------------------------------------------------- */
/* Bounded reader (crates/vocal-model/src/retrieval.rs:200-268)               */
/* ------------------------------------------------------------------------- */

typedef struct {
    const uint8_t *bytes;
    size_t len;
    size_t pos;
    char *err;
    size_t errlen;
} rd;

static int fail(rd *r, const char *msg) {
    if (r->err && r->errlen) snprintf(r->err, r->errlen, "RVC retrieval index: %s", msg);
    return -1;
}

static size_t remaining(const rd *r) { return r->len - r->pos; }

static int take(rd *r, size_t count, const uint8_t **out) {
    if (count > r->len - r->pos) return fail(r, "truncated index");
    *out = r->bytes + r->pos;
    r->pos += count;
    return 0;
}

static int tag(rd *r, uint8_t out[4]) {
    const uint8_t *p;
    if (take(r, 4, &p)) return -1;
    memcpy(out, p, 4);
    return 0;
}

static int rd_u64(rd *r, uint64_t *out) {
    const uint8_t *p;
    if (take(r, 8, &p)) return -1;
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
    *out = v;
    return 0;
}

static int skip_elements(rd *r, uint64_t count, uint64_t size) {
    const uint8_t *p;
    if (size && count > SIZE_MAX / size) return fail(r, "size overflow");
    return take(r, (size_t)(count * size), &p);
}

static int header(rd *r, uint64_t *d_out, uint64_t *count_out) {
    uint8_t t[4];
    uint64_t count;
    const uint8_t *p;
    if (tag(r, t)) return -1;
    int32_t d = (int32_t)((uint32_t)t[0] | (uint32_t)t[1] << 8 | (uint32_t)t[2] << 16 | (uint32_t)t[3] << 24);
    if (rd_u64(r, &count)) return -1;
    if (take(r, 16, &p)) return -1; /* legacy dummy fields */
    if (take(r, 1, &p)) return -1;
    uint8_t trained = p[0];
    if (tag(r, t)) return -1;
    int32_t metric = (int32_t)((uint32_t)t[0] | (uint32_t)t[1] << 8 | (uint32_t)t[2] << 16 | (uint32_t)t[3] << 24);
    if (!(d >= 1 && d <= 4096) || count == 0 || count > (uint64_t)INT32_MAX || trained != 1 || metric != 1)
        return fail(r, "requires a populated, trained L2 index, width <= 4096 and i32 row count");
    *d_out = (uint64_t)d;
    *count_out = count;
    return 0;
}

/* Reader::floats: optional u64 length prefix, then count little-endian f32
 * values that must all be finite.  *dst is malloc'd here, after the bytes
 * are known to be present (the reference bounds allocation the same way). */
static int floats(rd *r, uint64_t count, int length_prefix, float **dst) {
    if (length_prefix) {
        uint64_t n;
        if (rd_u64(r, &n)) return -1;
        if (n != count) return fail(r, "float vector length mismatch");
    }
    const uint8_t *p;
    if (count > SIZE_MAX / 4) return fail(r, "float shape overflow");
    if (take(r, (size_t)(count * 4), &p)) return -1;
    float *out = malloc((size_t)count * 4 + 4);
    if (!out) return fail(r, "out of memory");
    memcpy(out, p, (size_t)count * 4);
    for (uint64_t i = 0; i < count; ++i)
        if (!isfinite(out[i])) {
            free(out);
            return fail(r, "non-finite vector");
        }
    *dst = out;
    return 0;
}

void orc_free(orc_index *ix) {
    if (!ix) return;
    free(ix->centroids);
    free(ix->offsets);
    free(ix->vectors);
    free(ix->ids);
    memset(ix, 0, sizeof(*ix));
}

/* RetrievalIndex::from_faiss -- crates/vocal-model/src/retrieval.rs:62-193.
 * Returns 0 and fills *out, or -1 with a message in err. */
int orc_parse_faiss(const uint8_t *bytes, size_t len, orc_index *out, char *err, size_t errlen) {
    rd r = {bytes, len, 0, err, errlen};
    orc_index ix;
    memset(&ix, 0, sizeof(ix));
    memset(out, 0, sizeof(*out));
    uint8_t kind[4];
    uint64_t d, count;
    if (tag(&r, kind)) goto bad;
    if (header(&r, &d, &count)) goto bad;
    if (!memcmp(kind, "IxF2", 4)) {
        if (count > UINT64_MAX / d) { fail(&r, "shape overflow"); goto bad; }
        if (floats(&r, d * count, 1, &ix.vectors)) goto bad;
        ix.d = (int64_t)d;
        ix.nprobe = 1;
        ix.nlist = 1;
        ix.n = (int64_t)count;
        ix.centroids = calloc((size_t)d, 4);
        ix.offsets = malloc(2 * sizeof(int32_t));
        ix.ids = malloc((size_t)count * sizeof(int32_t));
        if (!ix.centroids || !ix.offsets || !ix.ids) { fail(&r, "out of memory"); goto bad; }
        ix.offsets[0] = 0;
        ix.offsets[1] = (int32_t)count;
        for (uint64_t i = 0; i < count; ++i) ix.ids[i] = (int32_t)i;
    } else if (!memcmp(kind, "IwFl", 4)) {
        uint64_t nlist, nprobe;
        if (rd_u64(&r, &nlist) || rd_u64(&r, &nprobe)) goto bad;
        if (nlist == 0 || nprobe == 0 || nprobe > nlist || nlist > len / 8) {
            fail(&r, "invalid IVF list/probe count");
            goto bad;
        }
        uint8_t t[4];
        if (tag(&r, t)) goto bad;
        if (memcmp(t, "IxF2", 4)) { fail(&r, "IVF requires a Flat-L2 coarse quantizer"); goto bad; }
        uint64_t cd, cc;
        if (header(&r, &cd, &cc)) goto bad;
        if (cd != d || cc != nlist) { fail(&r, "coarse quantizer shape mismatch"); goto bad; }
        if (nlist > UINT64_MAX / d) { fail(&r, "centroid shape overflow"); goto bad; }
        if (floats(&r, nlist * d, 1, &ix.centroids)) goto bad;
        const uint8_t *p;
        if (take(&r, 1, &p)) goto bad;
        uint8_t map_kind = p[0];
        uint64_t map_len;
        if (rd_u64(&r, &map_len)) goto bad;
        if (map_kind > 2 || (map_kind == 0 && map_len != 0) || (map_kind == 1 && map_len != count)) {
            fail(&r, "invalid direct map");
            goto bad;
        }
        if (skip_elements(&r, map_len, 8)) goto bad;
        if (map_kind == 2) {
            uint64_t hn;
            if (rd_u64(&r, &hn) || skip_elements(&r, hn, 16)) goto bad;
        }
        if (tag(&r, t)) goto bad;
        if (memcmp(t, "ilar", 4)) { fail(&r, "only ArrayInvertedLists is supported"); goto bad; }
        uint64_t il_n, code_size;
        if (rd_u64(&r, &il_n)) goto bad;
        if (il_n != nlist) { fail(&r, "inverted-list layout mismatch"); goto bad; }
        if (rd_u64(&r, &code_size)) goto bad;
        if (code_size != d * 4) { fail(&r, "inverted-list layout mismatch"); goto bad; }
        uint8_t sizes_kind[4];
        uint64_t sizes_len;
        if (tag(&r, sizes_kind) || rd_u64(&r, &sizes_len)) goto bad;
        uint64_t *sizes = calloc((size_t)nlist, sizeof(uint64_t));
        if (!sizes) { fail(&r, "out of memory"); goto bad; }
        if (!memcmp(sizes_kind, "full", 4) && sizes_len == nlist) {
            for (uint64_t l = 0; l < nlist; ++l)
                if (rd_u64(&r, &sizes[l])) { free(sizes); goto bad; }
        } else if (!memcmp(sizes_kind, "sprs", 4) && sizes_len % 2 == 0 && sizes_len / 2 <= nlist) {
            for (uint64_t e = 0; e < sizes_len / 2; ++e) {
                uint64_t list, size;
                if (rd_u64(&r, &list) || rd_u64(&r, &size)) { free(sizes); goto bad; }
                if (list >= nlist || size == 0 || sizes[list] != 0) {
                    free(sizes);
                    fail(&r, "invalid sparse list directory");
                    goto bad;
                }
                sizes[list] = size;
            }
        } else {
            free(sizes);
            fail(&r, "invalid inverted-list size directory");
            goto bad;
        }
        uint64_t total = 0;
        for (uint64_t l = 0; l < nlist; ++l) {
            if (sizes[l] > UINT64_MAX - total) { free(sizes); fail(&r, "list size overflow"); goto bad; }
            total += sizes[l];
        }
        if (total != count) { free(sizes); fail(&r, "list sizes disagree with ntotal"); goto bad; }
        if (count > UINT64_MAX / (d * 4 + 8)) { free(sizes); fail(&r, "payload overflow"); goto bad; }
        if (count * (d * 4 + 8) != remaining(&r)) { free(sizes); fail(&r, "truncated or trailing IVF payload"); goto bad; }
        ix.vectors = malloc((size_t)(count * d) * 4 + 4);
        ix.ids = malloc((size_t)count * sizeof(int32_t) + 4);
        ix.offsets = malloc((size_t)(nlist + 1) * sizeof(int32_t));
        uint8_t *seen = calloc((size_t)count, 1);
        if (!ix.vectors || !ix.ids || !ix.offsets || !seen) {
            free(sizes);
            free(seen);
            fail(&r, "out of memory");
            goto bad;
        }
        uint64_t filled = 0;
        ix.offsets[0] = 0;
        for (uint64_t l = 0; l < nlist; ++l) {
            float *chunk = NULL;
            if (floats(&r, sizes[l] * d, 0, &chunk)) { free(sizes); free(seen); goto bad; }
            memcpy(ix.vectors + filled * d, chunk, (size_t)(sizes[l] * d) * 4);
            free(chunk);
            for (uint64_t s = 0; s < sizes[l]; ++s) {
                uint64_t id;
                if (rd_u64(&r, &id)) { free(sizes); free(seen); goto bad; }
                if (id >= count || seen[id]) {
                    free(sizes);
                    free(seen);
                    fail(&r, "RVC requires unique IDs in 0..ntotal");
                    goto bad;
                }
                seen[id] = 1;
                ix.ids[filled + s] = (int32_t)id;
            }
            filled += sizes[l];
            ix.offsets[l + 1] = (int32_t)filled;
        }
        free(sizes);
        free(seen);
        ix.d = (int64_t)d;
        ix.nprobe = (int64_t)nprobe;
        ix.nlist = (int64_t)nlist;
        ix.n = (int64_t)count;
    } else {
        fail(&r, "supported FAISS types are IxF2 and IwFl (L2 Flat/IVFFlat)");
        goto bad;
    }
    if (remaining(&r) != 0) {
        fail(&r, "unexpected trailing data");
        goto bad;
    }
    *out = ix;
    return 0;
bad:
    orc_free(&ix);
    return -1;
}

/* ------------------------------------------------------------------------- */
/* VFRM aux.retrieval.faiss extraction                                        */
/* (crates/vocal-model/src/inspection.rs:70-178, retrieval.rs:45-57)          */
/* ------------------------------------------------------------------------- */

static uint64_t le64(const uint8_t *p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
    return v;
}
static uint32_t le32(const uint8_t *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}

/* Locates the U8 tensor `aux.retrieval.faiss` in a VFRM v1 image.
 * Returns 1 with (*off, *n) set when present, 0 when absent, -1 when the
 * container is malformed.  JSON manifest validation is not restated. */
int orc_vfrm_find_faiss(const uint8_t *b, size_t len, uint64_t *off, uint64_t *n) {
    static const uint8_t magic[8] = {'V', 'F', 'R', 'M', 0, 0, 0, 1};
    if (len < 64 || memcmp(b, magic, 8)) return -1;
    uint32_t header_size = le32(b + 12);
    uint64_t meta_len = le64(b + 16), count = le64(b + 24), dir_len = le64(b + 32), data_off = le64(b + 40);
    if (header_size != 64 || meta_len > len || dir_len > len) return -1;
    uint64_t dir_off = 64 + meta_len, dir_end = dir_off + dir_len;
    if (dir_end > len || data_off < dir_end || data_off > len) return -1;
    const uint8_t *dp = b + dir_off;
    uint64_t pos = 0;
    int found = 0;
    for (uint64_t t = 0; t < count; ++t) {
        if (pos + 8 > dir_len) return -1;
        uint32_t name_len = le32(dp + pos);
        uint8_t dtype = dp[pos + 4], rank = dp[pos + 5];
        pos += 8;
        if (name_len == 0 || name_len > 65535 || rank > 64 || dtype < 1 || dtype > 6) return -1;
        if (pos + name_len + 8ull * rank + 16 > dir_len) return -1;
        const uint8_t *name = dp + pos;
        pos += name_len;
        static const uint64_t esize[7] = {0, 1, 4, 8, 2, 4, 2};
        uint64_t expected = esize[dtype];
        uint64_t dim0 = 0;
        for (uint32_t k = 0; k < rank; ++k) {
            uint64_t dim = le64(dp + pos + 8ull * k);
            if (k == 0) dim0 = dim;
            if (dim && expected > UINT64_MAX / dim) return -1;
            expected *= dim;
        }
        pos += 8ull * rank;
        uint64_t toff = le64(dp + pos), tlen = le64(dp + pos + 8);
        pos += 16;
        if (expected != tlen || toff < data_off || toff > len || tlen > len - toff) return -1;
        if (name_len == 19 && !memcmp(name, "aux.retrieval.faiss", 19)) {
            if (dtype != 1 || rank != 1 || dim0 != tlen) return -1;
            *off = toff;
            *n = tlen;
            found = 1;
        }
    }
    if (pos != dir_len) return -1;
    return found;
}

/* ------------------------------------------------------------------------- */
/* Distances (crates/vocal-cpu/src/retrieval.rs:5-26)                         */
/* ------------------------------------------------------------------------- */

/* scalar_l2: sequential fold of (a-b)*(a-b), starting from -0.0. */
float orc_l2_scalar(const float *a, const float *b, size_t d) {
    float s = -0.0f;
    for (size_t i = 0; i < d; ++i) {
        float t = a[i] - b[i];
        s = s + t * t;
    }
    return s;
}

/* avx2_l2: 8-lane sum += (a-b)*(a-b) (mul and add separate), lanes folded
 * 0..7 from -0.0, then + scalar_l2 of the tail. */
__attribute__((target("avx2"))) float orc_l2_avx2(const float *a, const float *b, size_t d) {
    __m256 sum = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= d) {
        __m256 delta = _mm256_sub_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i));
        sum = _mm256_add_ps(sum, _mm256_mul_ps(delta, delta));
        i += 8;
    }
    float lanes[8];
    _mm256_storeu_ps(lanes, sum);
    float s = -0.0f;
    for (int l = 0; l < 8; ++l) s = s + lanes[l];
    return s + orc_l2_scalar(a + i, b + i, d - i);
}

/* Portable restatement of the AVX2 order without intrinsics; must agree
 * bit-for-bit with orc_l2_avx2 (checked by the tests). */
float orc_l2_lanes(const float *a, const float *b, size_t d) {
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    while (i + 8 <= d) {
        for (int l = 0; l < 8; ++l) {
            float t = a[i + l] - b[i + l];
            lanes[l] = lanes[l] + t * t;
        }
        i += 8;
    }
    float s = -0.0f;
    for (int l = 0; l < 8; ++l) s = s + lanes[l];
    return s + orc_l2_scalar(a + i, b + i, d - i);
}

typedef float (*dist_fn)(const float *, const float *, size_t);

/* f32::total_cmp as a signed-integer key. */
static int32_t total_key(float f) {
    int32_t x;
    memcpy(&x, &f, 4);
    return x ^ (int32_t)(((uint32_t)(x >> 31)) >> 1);
}

typedef struct {
    float dist;
    int64_t id;
} orc_pair;

static int coarse_cmp(const void *pa, const void *pb) {
    const orc_pair *a = pa, *b = pb;
    int32_t ka = total_key(a->dist), kb = total_key(b->dist);
    if (ka != kb) return ka < kb ? -1 : 1;
    return a->id < b->id ? -1 : (a->id > b->id);
}

/* The search half of blend (crates/vocal-cpu/src/retrieval.rs:45-65):
 * coarse scan + sort by (dist total_cmp, list id), first nprobe lists in
 * order, rows in storage order, insertion top-8 where ties keep the earlier
 * scanned row.  Writes best[8] (storage rows, -1 when empty) and returns the
 * filled count.  `probe_override` > 0 replaces the persisted nprobe. */
static int search_row(const orc_index *ix, const float *row, dist_fn distance, int64_t nprobe,
                      orc_pair *lists, float best_d[ORC_K], int64_t best_i[ORC_K]) {
    const size_t d = (size_t)ix->d;
    for (int64_t l = 0; l < ix->nlist; ++l) {
        lists[l].dist = distance(row, ix->centroids + (size_t)l * d, d);
        lists[l].id = l;
    }
    qsort(lists, (size_t)ix->nlist, sizeof(orc_pair), coarse_cmp);
    for (int k = 0; k < ORC_K; ++k) {
        best_d[k] = INFINITY;
        best_i[k] = -1;
    }
    for (int64_t p = 0; p < nprobe && p < ix->nlist; ++p) {
        int64_t list = lists[p].id;
        for (int64_t id = ix->offsets[list]; id < ix->offsets[list + 1]; ++id) {
            float score = distance(row, ix->vectors + (size_t)id * d, d);
            if (score >= best_d[ORC_K - 1]) continue;
            int pos = 0;
            while (pos < ORC_K && best_d[pos] <= score) ++pos; /* partition_point(v <= score) */
            for (int k = ORC_K - 1; k > pos; --k) {
                best_d[k] = best_d[k - 1];
                best_i[k] = best_i[k - 1];
            }
            best_d[pos] = score;
            best_i[pos] = id;
        }
    }
    int count = 0;
    while (count < ORC_K && best_i[count] != -1) ++count;
    return count;
}

/* The weights + blend half (crates/vocal-cpu/src/retrieval.rs:65-81). */
static void blend_from_best(const orc_index *ix, float *row, float ratio, int count, const float best_d[ORC_K],
                            const int64_t best_i[ORC_K]) {
    const size_t d = (size_t)ix->d;
    double w[ORC_K] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < count; ++k) {
        float s = best_d[k] > 1e-12f ? best_d[k] : 1e-12f; /* f32::max(score, 1e-12) */
        if (isnan(best_d[k])) s = 1e-12f;
        double sd = (double)s;
        w[k] = 1.0 / (sd * sd);
    }
    double sum = -0.0;
    for (int k = 0; k < ORC_K; ++k) sum = sum + w[k];
    for (size_t j = 0; j < d; ++j) {
        double acc = -0.0;
        for (int k = 0; k < count; ++k) {
            double t = (double)ix->vectors[(size_t)best_i[k] * d + j] * w[k];
            t = t / sum;
            acc = acc + t;
        }
        float retrieved = (float)acc;
        float a = row[j] * (1.0f - ratio);
        float b = retrieved * ratio;
        row[j] = a + b;
    }
}

/* Status codes of the per-frame oracle. */
#define ORC_OK 0
#define ORC_ERR_CONFIG 1       /* "invalid retrieval dimensions or empty index" */
#define ORC_ERR_NO_CANDIDATE 2 /* "IVF search selected no candidate" */

/* crates/vocal-cpu/src/retrieval.rs:27-83 for one row (in place). */
int orc_blend_row(const orc_index *ix, float *row, int64_t d, float ratio, int simd) {
    if (d != ix->d || ix->n == 0) return ORC_ERR_CONFIG;
    orc_pair *lists = malloc((size_t)ix->nlist * sizeof(orc_pair));
    if (!lists) return ORC_ERR_CONFIG;
    float bd[ORC_K];
    int64_t bi[ORC_K];
    int count = search_row(ix, row, simd ? orc_l2_avx2 : orc_l2_scalar, ix->nprobe, lists, bd, bi);
    free(lists);
    if (count == 0) return ORC_ERR_NO_CANDIDATE;
    blend_from_best(ix, row, ratio, count, bd, bi);
    return ORC_OK;
}

/* Search only: top-8 squared distances, storage rows and FAISS labels
 * (ids[row]); unfilled slots get +inf / -1 / -1.  Returns the count. */
int orc_search_row(const orc_index *ix, const float *row, int simd, int64_t nprobe, float *dist8, int64_t *rows8,
                   int64_t *labels8) {
    orc_pair *lists = malloc((size_t)ix->nlist * sizeof(orc_pair));
    if (!lists) return -1;
    float bd[ORC_K];
    int64_t bi[ORC_K];
    int count = search_row(ix, row, simd ? orc_l2_avx2 : orc_l2_scalar, nprobe > 0 ? nprobe : ix->nprobe, lists,
                           bd, bi);
    free(lists);
    for (int k = 0; k < ORC_K; ++k) {
        dist8[k] = bd[k];
        rows8[k] = bi[k];
        labels8[k] = bi[k] >= 0 ? ix->ids[bi[k]] : -1;
    }
    return count;
}

/* Batch driver: the reference call site (crates/vocal-cpu/src/pipeline.rs:
 * 292-301) loops serially over frames; `threads` > 1 splits frames across
 * POSIX threads for the all-cores baseline.  ratio <= 0 skips the blend like
 * the call site.  status[f] receives the per-frame code (may be NULL). */
typedef struct {
    const orc_index *ix;
    float *feats;
    int64_t d;
    float ratio;
    int simd;
    int32_t *status;
    int64_t begin, end;
} job;

static void *run_job(void *p) {
    job *j = p;
    for (int64_t f = j->begin; f < j->end; ++f) {
        int rc = orc_blend_row(j->ix, j->feats + f * j->d, j->d, j->ratio, j->simd);
        if (j->status) j->status[f] = rc;
    }
    return NULL;
}

int orc_blend_batch(const orc_index *ix, float *feats, int64_t frames, int64_t d, float ratio, int simd, int threads,
                    int32_t *status) {
    if (!(ratio > 0.0f)) {
        if (status)
            for (int64_t f = 0; f < frames; ++f) status[f] = ORC_OK;
        return 0;
    }
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > frames) threads = (int)(frames > 0 ? frames : 1);
    pthread_t tid[256];
    job jobs[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (job){ix, feats, d, ratio, simd, status, frames * t / threads, frames * (t + 1) / threads};
        if (t > 0) pthread_create(&tid[t], NULL, run_job, &jobs[t]);
    }
    run_job(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
    int bad = 0;
    if (status)
        for (int64_t f = 0; f < frames; ++f) bad += status[f] != ORC_OK;
    return bad;
}

/* Batch search (threads as above).  Outputs are [frames][8]. */
typedef struct {
    const orc_index *ix;
    const float *q;
    int simd;
    int64_t nprobe;
    float *dist;
    int64_t *rows, *labels;
    int32_t *count;
    int64_t begin, end;
} sjob;

static void *run_sjob(void *p) {
    sjob *j = p;
    for (int64_t f = j->begin; f < j->end; ++f) {
        int c = orc_search_row(j->ix, j->q + f * j->ix->d, j->simd, j->nprobe, j->dist + f * ORC_K,
                               j->rows + f * ORC_K, j->labels + f * ORC_K);
        if (j->count) j->count[f] = c;
    }
    return NULL;
}

int orc_search_batch(const orc_index *ix, const float *q, int64_t frames, int simd, int64_t nprobe, int threads,
                     float *dist, int64_t *rows, int64_t *labels, int32_t *count) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > frames) threads = (int)(frames > 0 ? frames : 1);
    pthread_t tid[256];
    sjob jobs[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (sjob){ix, q, simd, nprobe, dist, rows, labels, count, frames * t / threads,
                         frames * (t + 1) / threads};
        if (t > 0) pthread_create(&tid[t], NULL, run_sjob, &jobs[t]);
    }
    run_sjob(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
    return 0;
}

/* Wraps caller-owned arrays as an index without copying (for synthetic data
 * that never went through FAISS bytes).  orc_free must not be called on it. */
void orc_view(orc_index *ix, int64_t d, int64_t nlist, int64_t nprobe, int64_t n, float *centroids, int32_t *offsets,
              float *vectors, int32_t *ids) {
    ix->d = d;
    ix->nlist = nlist;
    ix->nprobe = nprobe;
    ix->n = n;
    ix->centroids = centroids;
    ix->offsets = offsets;
    ix->vectors = vectors;
    ix->ids = ids;
}

size_t orc_index_size(void) { return sizeof(orc_index); }

/* Unvoiced-frame protection, restating protect_features
 * (crates/vocal-tensorrt/native/retrieval_protection.cu:4-16) element by
 * element: nothing when ratio <= 0 or protect >= 0.5 (NaN passes both); frames
 * with pitchf > 0 keep their features; the others become
 * f * p + raw[min(frame / 2, hubert_frames - 1)] * (1 - p), each operation
 * rounded on its own (this file builds with -ffp-contract=off). */
void orc_protect(float *features, const float *raw, const float *pitchf, float ratio, float protect,
                 int64_t frames, int64_t hubert_frames, int64_t width) {
    if (ratio <= 0.0f || protect >= 0.5f) return;
    for (int64_t f = 0; f < frames; ++f) {
        if (pitchf[f] > 0.0f) continue;
        const int64_t row = f / 2 < hubert_frames - 1 ? f / 2 : hubert_frames - 1;
        for (int64_t c = 0; c < width; ++c) {
            const float a = features[f * width + c] * protect;
            const float b = raw[row * width + c] * (1.0f - protect);
            features[f * width + c] = a + b;
        }
    }
}

/* The RVC frontend after the blend with the protection fused, restating
 * frontend.cpp:36-75 (a TensorRT graph in the reference) then protect_features:
 * target = min(2 (hubert_frames + 1), f0_frames); output frame t reads HuBERT
 * row min(t / 2, hubert_frames - 1) (the appended last frame and the nearest,
 * asymmetric 2x resize); pitchf = f0[t]; coarse[t] = the unrounded mel bin
 * (before clamping) and pitch[t] its clamped, rounded (half to even) value.
 * raw == NULL skips the protection.  Returns target. */
int64_t orc_rvc_frontend(const float *hubert, const float *raw, const float *f0, float ratio, float protect,
                         int64_t hubert_frames, int64_t f0_frames, int64_t width, float *feats, float *pitchf,
                         int32_t *pitch, float *coarse) {
    const int64_t interp = 2 * (hubert_frames + 1);
    const int64_t target = interp < f0_frames ? interp : f0_frames;
    const int protecting = raw != NULL && !(ratio <= 0.0f || protect >= 0.5f);
    const float mel_min = 1127.0f * log1pf(50.0f / 700.0f);
    const float mel_max = 1127.0f * log1pf(1100.0f / 700.0f);
    const float mel_scale = 254.0f / (mel_max - mel_min);
    for (int64_t t = 0; t < target; ++t) {
        const int64_t row = t / 2 < hubert_frames - 1 ? t / 2 : hubert_frames - 1;
        const float f = f0[t];
        for (int64_t c = 0; c < width; ++c) {
            float v = hubert[row * width + c];
            if (protecting && !(f > 0.0f)) {
                const float a = v * protect;
                const float b = raw[row * width + c] * (1.0f - protect);
                v = a + b;
            }
            feats[t * width + c] = v;
        }
        pitchf[t] = f;
        const float scaled = f * (1.0f / 700.0f);
        const float mel = logf(scaled + 1.0f) * 1127.0f;
        float x = (mel - mel_min) * mel_scale + 1.0f;
        if (coarse) coarse[t] = x;
        x = x > 1.0f ? x : 1.0f;
        x = x < 255.0f ? x : 255.0f;
        pitch[t] = (int32_t)rintf(x);
    }
    return target;
}

/* The generic engine's frontend, restating crates/vocal-engine/src/
 * pipeline.rs: interpolate_2x (75-96) of the blended features into
 * out[2 frames][width]; when hz != NULL, raw != NULL and protect < 0.5
 * (313), the protection (321-333) over t < min(2 frames, hz_frames) against
 * interpolate_2x of raw; coarse[t] = f0_to_coarse(hz[t]) (625-633) for the
 * same frames when hz != NULL.  Returns the number of coarse values. */
static float orc_lerp_half(float a, float b, float w) {
    const float x = a * (1.0f - w);
    const float y = b * w;
    return x + y;
}

static int32_t orc_f0_to_coarse(float f0, float mel_min, float mel_max) {
    if (f0 <= 0.0f) return 1;
    const float mel = 1127.0f * logf(1.0f + f0 / 700.0f);
    const float scaled = (mel - mel_min) * 254.0f;
    const float r = roundf(scaled / (mel_max - mel_min) + 1.0f);
    if (r != r) return 0; /* Rust: clamp keeps NaN, `as i32` saturates NaN to 0 */
    const float c = r < 1.0f ? 1.0f : (r > 255.0f ? 255.0f : r);
    return (int32_t)c;
}

int64_t orc_engine_frontend(const float *blended, const float *raw, const float *hz, float protect, int64_t frames,
                            int64_t hz_frames, int64_t width, float *out, int32_t *coarse) {
    const int64_t out_frames = 2 * frames;
    const int64_t pitch_frames = hz == NULL ? 0 : (hz_frames < out_frames ? hz_frames : out_frames);
    const int mixing = hz != NULL && raw != NULL && protect < 0.5f;
    const float p = protect < 0.0f ? 0.0f : (protect > 1.0f ? 1.0f : protect);
    const float mel_min = 1127.0f * logf(1.0f + 50.0f / 700.0f);
    const float mel_max = 1127.0f * logf(1.0f + 1100.0f / 700.0f);
    for (int64_t t = 0; t < out_frames; ++t) {
        const float source = (float)t / 2.0f;
        const int64_t left = (int64_t)floorf(source);
        const int64_t right = left + 1 < frames ? left + 1 : frames - 1;
        const float w = source - (float)left;
        const int mix = mixing && t < pitch_frames;
        const float v = mix ? (hz[t] > 0.0f ? 1.0f : p) : 1.0f;
        for (int64_t c = 0; c < width; ++c) {
            float f = orc_lerp_half(blended[left * width + c], blended[right * width + c], w);
            if (mix) {
                const float before = orc_lerp_half(raw[left * width + c], raw[right * width + c], w);
                const float a = f * v;
                const float b = before * (1.0f - v);
                f = a + b;
            }
            out[t * width + c] = f;
        }
        if (hz != NULL && t < pitch_frames) coarse[t] = orc_f0_to_coarse(hz[t], mel_min, mel_max);
    }
    return pitch_frames;
}

/* ---------------------------------------------------------------- IVF trainer */

static uint64_t orc_splitmix(uint64_t *state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static float orc_uniform(uint64_t *state) { return (float)(orc_splitmix(state) >> 40) * 0x1p-24f; }

/* the first m entries of a Fisher-Yates shuffle of 0..n-1 */
static int orc_shuffled_prefix(int64_t n, int64_t m, uint64_t seed, int64_t *out) {
    int64_t *p = (int64_t *)malloc((size_t)n * sizeof(int64_t));
    if (!p) return -1;
    for (int64_t i = 0; i < n; ++i) p[i] = i;
    uint64_t st = seed;
    for (int64_t i = 0; i < m; ++i) {
        const int64_t j = i + (int64_t)(orc_splitmix(&st) % (uint64_t)(n - i));
        const int64_t t = p[i];
        p[i] = p[j];
        p[j] = t;
    }
    memcpy(out, p, (size_t)m * sizeof(int64_t));
    free(p);
    return 0;
}

/* nearest centroid under avx2_l2's order, ties to the lower centroid */
static int32_t orc_nearest(const float *c, int32_t k, const float *row, int32_t d, float *dist) {
    int32_t best = 0;
    float bd = orc_l2_lanes(row, c, (size_t)d);
    for (int32_t j = 1; j < k; ++j) {
        const float v = orc_l2_lanes(row, c + (size_t)j * d, (size_t)d);
        if (v < bd) {
            bd = v;
            best = j;
        }
    }
    *dist = bd;
    return best;
}

typedef struct {
    const float *c, *x;
    int32_t k, d;
    int64_t lo, hi;
    int32_t *lists;
    float *dist;
} assign_job;

static void *run_assign(void *p) {
    assign_job *j = (assign_job *)p;
    for (int64_t r = j->lo; r < j->hi; ++r) j->lists[r] = orc_nearest(j->c, j->k, j->x + r * j->d, j->d, &j->dist[r]);
    return NULL;
}

void orc_ivf_assign(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t *lists,
                    float *dist, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    assign_job jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (assign_job){centroids, x, k, d, n * t / threads, n * (t + 1) / threads, lists, dist};
        if (t > 0) pthread_create(&tid[t], NULL, run_assign, &jobs[t]);
    }
    run_assign(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
}

/* Restates vfr_kmeans (see the header comment); returns 0, or -1 on bad
 * arguments / allocation failure. */
int orc_kmeans(const float *x, int64_t n, int32_t d, int32_t k, int32_t niter, int32_t max_ppc, uint64_t seed,
               float *centroids, double *objective, int threads) {
    if (!x || !centroids || d <= 0 || k <= 0 || n < k || niter < 0 || max_ppc < 0) return -1;
    int64_t m = n;
    if (max_ppc > 0 && n > (int64_t)k * max_ppc) m = (int64_t)k * max_ppc;
    float *train = (float *)x;
    float *sample = NULL;
    int64_t *rows = (int64_t *)malloc((size_t)(m > k ? m : k) * sizeof(int64_t));
    int32_t *lists = (int32_t *)malloc((size_t)m * sizeof(int32_t));
    float *dist = (float *)malloc((size_t)m * sizeof(float));
    int64_t *sums = (int64_t *)malloc((size_t)k * d * sizeof(int64_t));
    long long *counts = (long long *)malloc((size_t)k * sizeof(long long));
    double *w = (double *)malloc((size_t)k * sizeof(double));
    if (!rows || !lists || !dist || !sums || !counts || !w) goto fail;
    if (m < n) {
        sample = (float *)malloc((size_t)m * d * sizeof(float));
        if (!sample || orc_shuffled_prefix(n, m, seed, rows)) goto fail;
        for (int64_t i = 0; i < m; ++i) memcpy(sample + i * d, x + rows[i] * d, (size_t)d * sizeof(float));
        train = sample;
    }
    if (orc_shuffled_prefix(m, k, seed + 1, rows)) goto fail;
    for (int32_t j = 0; j < k; ++j) memcpy(centroids + (size_t)j * d, train + rows[j] * d, (size_t)d * sizeof(float));
    float maxabs = 0.0f;
    for (int64_t i = 0; i < m * d; ++i) {
        const float a = fabsf(train[i]);
        if (a > maxabs) maxabs = a;
    }
    int e = 0;
    frexpf(maxabs, &e);
    int bits = 0;
    while (((int64_t)1 << bits) < m) ++bits;
    const int sexp = 62 - bits - e;
    const double scale = ldexp(1.0, sexp), inv = ldexp(1.0, -sexp);
    uint64_t split = seed + 2;
    for (int32_t it = 0; it < niter; ++it) {
        orc_ivf_assign(centroids, k, train, m, d, lists, dist, threads);
        double obj = 0.0;
        for (int64_t r = 0; r < m; ++r) obj += dist[r];
        if (objective) objective[it] = obj;
        memset(sums, 0, (size_t)k * d * sizeof(int64_t));
        memset(counts, 0, (size_t)k * sizeof(long long));
        for (int64_t r = 0; r < m; ++r) {
            const int32_t l = lists[r];
            ++counts[l];
            for (int32_t c = 0; c < d; ++c) sums[(size_t)l * d + c] += llrint((double)train[r * d + c] * scale);
        }
        int empty = 0;
        for (int32_t j = 0; j < k; ++j) {
            empty |= counts[j] == 0;
            for (int32_t c = 0; c < d; ++c)
                centroids[(size_t)j * d + c] =
                    counts[j] > 0 ? (float)(((double)sums[(size_t)j * d + c] / (double)counts[j]) * inv) : 0.0f;
        }
        if (!empty) continue;
        for (int32_t j = 0; j < k; ++j) w[j] = (double)counts[j];
        for (int32_t ci = 0; ci < k; ++ci) {
            if (w[ci] != 0.0) continue;
            int32_t cj = 0;
            int found = 0;
            const long long trials = 64LL * k + 1024;
            for (long long t = 0; t < trials; ++t, cj = (cj + 1) % k) {
                const double p = (w[cj] - 1.0) / (double)(m - k);
                if ((double)orc_uniform(&split) < p) {
                    found = 1;
                    break;
                }
            }
            if (!found) {
                cj = 0;
                for (int32_t j = 1; j < k; ++j)
                    if (w[j] > w[cj]) cj = j;
            }
            float *a = centroids + (size_t)ci * d, *b = centroids + (size_t)cj * d;
            memcpy(a, b, (size_t)d * sizeof(float));
            for (int32_t j = 0; j < d; ++j) {
                if (j % 2 == 0) {
                    a[j] *= 1.0f + 1.0f / 1024.0f;
                    b[j] *= 1.0f - 1.0f / 1024.0f;
                } else {
                    a[j] *= 1.0f - 1.0f / 1024.0f;
                    b[j] *= 1.0f + 1.0f / 1024.0f;
                }
            }
            w[ci] = w[cj] / 2.0;
            w[cj] -= w[ci];
        }
    }
    free(sample);
    free(rows);
    free(lists);
    free(dist);
    free(sums);
    free(counts);
    free(w);
    return 0;
fail:
    free(sample);
    free(rows);
    free(lists);
    free(dist);
    free(sums);
    free(counts);
    free(w);
    return -1;
}
