// IVF training on the device: k-means for the coarse centroids, list
// assignment, a device index built straight from the assignment, and the
// FAISS IndexIVFFlat writer.
//
// The reference trains its indexes offline with FAISS
// (IndexIVFFlat::train, the recipe in crates/vocal-directml/tests/fixtures/
// README.md and scripts/benchmark-retrieval.py:56-65): Lloyd's k-means on at
// most k * max_points_per_centroid sampled rows, k sampled rows as the first
// centroids, empty clusters re-seeded by splitting a populated one with a
// small symmetric perturbation, then every row added to the list of its
// nearest centroid.  This trainer follows that algorithm with its own
// deterministic generator (SplitMix64) and three choices that make it
// reproducible bit for bit by the CPU restatement in oracle/vfr_oracle.c:
//   - assignment is the exact nearest centroid under the retrieval path's
//     own squared-L2 order (the engine's k=1 search), ties to the lower
//     centroid, so each row lands in the list its own probe ranks first;
//   - centroid sums are 64-bit fixed point (order independent);
//   - the split uses SplitMix64 draws in FAISS's visiting order.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

#include "index_build.h"
#include "kernels.h"
#include "tc_path.h"

namespace vfr {
namespace {

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014).
struct SplitMix {
    uint64_t state;
    uint64_t next() {
        uint64_t z = (state += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    float uniform() { return static_cast<float>(next() >> 40) * 0x1p-24f; }
};

// The first m entries of a Fisher-Yates shuffle of 0..n-1.
std::vector<int64_t> shuffled_prefix(int64_t n, int64_t m, uint64_t seed) {
    std::vector<int64_t> p(static_cast<size_t>(n));
    std::iota(p.begin(), p.end(), int64_t(0));
    SplitMix rng{seed};
    for (int64_t i = 0; i < m; ++i) {
        const int64_t j = i + static_cast<int64_t>(rng.next() % static_cast<uint64_t>(n - i));
        std::swap(p[i], p[j]);
    }
    p.resize(static_cast<size_t>(m));
    return p;
}

template <class T>
struct DeviceBuffer {
    T *p = nullptr;
    explicit DeviceBuffer(size_t count) {
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&p), std::max<size_t>(count, 1) * sizeof(T)), "cudaMalloc");
    }
    ~DeviceBuffer() {
        if (p) cudaFree(p);
    }
    DeviceBuffer(const DeviceBuffer &) = delete;
    DeviceBuffer &operator=(const DeviceBuffer &) = delete;
};

struct OwnedStream {
    cudaStream_t s = nullptr;
    OwnedStream() { cuda_check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)); }
    ~OwnedStream() {
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    }
};

constexpr size_t kSearchChunk = 32768;
constexpr float kSplitEps = 1.0f / 1024.0f;

// A flat index over k device rows (copied), labels 0..k-1.
VfrIndex *flat_index(const float *rows, int32_t k, int32_t d) {
    const VfrOptions o = resolve_options(nullptr);
    const std::vector<int32_t> offsets = {0, k};
    VfrIndex *ix = new_handle(d, 1, 1, static_cast<size_t>(k), offsets.data(), o);
    try {
        std::vector<int32_t> ids(static_cast<size_t>(k));
        std::iota(ids.begin(), ids.end(), 0);
        const std::vector<float> zero(static_cast<size_t>(d), 0.f);
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->centroids), zero.size() * sizeof(float)));
        cuda_check(cudaMemcpy(ix->centroids, zero.data(), zero.size() * sizeof(float), cudaMemcpyHostToDevice));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->offsets), offsets.size() * sizeof(int32_t)));
        cuda_check(cudaMemcpy(ix->offsets, offsets.data(), offsets.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        for (int32_t **dst : {&ix->ids, &ix->row_of_id}) {
            cuda_check(cudaMalloc(reinterpret_cast<void **>(dst), ids.size() * sizeof(int32_t)));
            cuda_check(cudaMemcpy(*dst, ids.data(), ids.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        }
        const size_t bytes = static_cast<size_t>(k) * d * sizeof(float);
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->vectors), bytes));
        cuda_check(cudaMemcpy(ix->vectors, rows, bytes, cudaMemcpyDeviceToDevice));
        finish_index(ix, o);
    } catch (...) {
        free_index(ix);
        throw;
    }
    return ix;
}

// Exact nearest centroid of each row: (distance, centroid) per row.
void nearest(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, float *dist, int64_t *labels,
             cudaStream_t s) {
    VfrIndex *ix = flat_index(centroids, k, d);
    try {
        for (int64_t off = 0; off < n; off += static_cast<int64_t>(kSearchChunk)) {
            const size_t len = static_cast<size_t>(std::min<int64_t>(static_cast<int64_t>(kSearchChunk), n - off));
            search_rows(ix, x + off * d, len, 1, dist + off, labels + off, s);
        }
        cuda_check(cudaStreamSynchronize(s));
    } catch (...) {
        cudaStreamSynchronize(s);
        free_index(ix);
        throw;
    }
    free_index(ix);
}

// 2^s with |x| 2^s < 2^(62 - ceil(log2 m)) for every |x| <= maxabs, so the
// sum of m such values fits an int64.
int fixed_point_exponent(float maxabs, int64_t m) {
    int e = 0;
    std::frexp(maxabs, &e);  // maxabs < 2^e (e = 0 for 0)
    int bits = 0;
    while ((int64_t(1) << bits) < m) ++bits;
    return 62 - bits - e;
}

// Clustering's empty-cluster split, visiting clusters in order: a donor cj
// is drawn by cycling from 0 with probability (w[cj] - 1) / (m - k), its
// centroid copied and both pushed apart by 1 +- 1/1024 (alternating by
// coordinate), its weight halved between the two.
void split_empty(std::vector<float> &c, std::vector<double> &w, int32_t k, int32_t d, int64_t m, SplitMix &rng) {
    for (int32_t ci = 0; ci < k; ++ci) {
        if (w[ci] != 0.0) continue;
        int32_t cj = 0;
        bool found = false;
        const long long trials = 64LL * k + 1024;
        for (long long t = 0; t < trials; ++t, cj = (cj + 1) % k) {
            const double p = (w[cj] - 1.0) / static_cast<double>(m - k);
            if (static_cast<double>(rng.uniform()) < p) {
                found = true;
                break;
            }
        }
        if (!found) cj = static_cast<int32_t>(std::max_element(w.begin(), w.end()) - w.begin());
        float *a = c.data() + static_cast<size_t>(ci) * d;
        float *b = c.data() + static_cast<size_t>(cj) * d;
        std::memcpy(a, b, static_cast<size_t>(d) * sizeof(float));
        for (int32_t j = 0; j < d; ++j) {
            if (j % 2 == 0) {
                a[j] *= 1.0f + kSplitEps;
                b[j] *= 1.0f - kSplitEps;
            } else {
                a[j] *= 1.0f - kSplitEps;
                b[j] *= 1.0f + kSplitEps;
            }
        }
        w[ci] = w[cj] / 2.0;
        w[cj] -= w[ci];
    }
}

void check_training_input(const float *x, int64_t n, int32_t d, int sms) {
    const unsigned long long bad = first_nonfinite(x, static_cast<unsigned long long>(n) * d, sms);
    require(bad == ~0ull, "non-finite training vector");
}

int device_sms() {
    int dev = 0, sms = 0;
    cuda_check(cudaGetDevice(&dev));
    cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return sms;
}

}  // namespace

void kmeans(const float *x, int64_t n, int32_t d, int32_t k, int32_t niter, int32_t max_points_per_centroid,
            uint64_t seed, float *centroids, double *objective, cudaStream_t stream) {
    require(x && centroids && d > 0 && d <= 4096 && k > 0 && n > 0 && n <= INT32_MAX && niter >= 0 &&
                max_points_per_centroid >= 0,
            "invalid k-means arguments");
    require(n >= k, "number of training points should be at least as large as number of clusters");
    const int sms = device_sms();
    check_training_input(x, n, d, sms);
    int64_t m = n;
    if (max_points_per_centroid > 0 && n > static_cast<int64_t>(k) * max_points_per_centroid)
        m = static_cast<int64_t>(k) * max_points_per_centroid;
    DeviceBuffer<float> sample(m < n ? static_cast<size_t>(m) * d : 0);
    const float *train = x;
    if (m < n) {
        const std::vector<int64_t> rows = shuffled_prefix(n, m, seed);
        DeviceBuffer<int64_t> dev_rows(rows.size());
        cuda_check(cudaMemcpy(dev_rows.p, rows.data(), rows.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
        launch_gather_rows(x, dev_rows.p, m, d, sample.p, stream);
        cuda_check(cudaStreamSynchronize(stream));
        train = sample.p;
    }
    {
        const std::vector<int64_t> first = shuffled_prefix(m, k, seed + 1);
        DeviceBuffer<int64_t> dev_first(first.size());
        cuda_check(cudaMemcpy(dev_first.p, first.data(), first.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
        launch_gather_rows(train, dev_first.p, k, d, centroids, stream);
        cuda_check(cudaStreamSynchronize(stream));
    }
    const int e = fixed_point_exponent(max_abs(train, static_cast<size_t>(m) * d), m);
    const double scale = std::ldexp(1.0, e), inv_scale = std::ldexp(1.0, -e);
    DeviceBuffer<float> dist(static_cast<size_t>(m));
    DeviceBuffer<int64_t> labels(static_cast<size_t>(m));
    DeviceBuffer<unsigned long long> sums(static_cast<size_t>(k) * d);
    DeviceBuffer<long long> dev_counts(static_cast<size_t>(k));
    std::vector<float> host_dist(static_cast<size_t>(m));
    std::vector<int64_t> host_labels(static_cast<size_t>(m));
    std::vector<long long> counts(static_cast<size_t>(k));
    std::vector<float> host_centroids;
    SplitMix split_rng{seed + 2};
    for (int32_t it = 0; it < niter; ++it) {
        nearest(centroids, k, train, m, d, dist.p, labels.p, stream);
        cuda_check(cudaMemcpy(host_dist.data(), dist.p, host_dist.size() * sizeof(float), cudaMemcpyDeviceToHost));
        cuda_check(
            cudaMemcpy(host_labels.data(), labels.p, host_labels.size() * sizeof(int64_t), cudaMemcpyDeviceToHost));
        double obj = 0.0;
        for (float v : host_dist) obj += v;
        if (objective) objective[it] = obj;
        std::fill(counts.begin(), counts.end(), 0LL);
        for (int64_t l : host_labels) {
            require(l >= 0 && l < k, "k-means assignment out of range");
            ++counts[static_cast<size_t>(l)];
        }
        cuda_check(cudaMemcpy(dev_counts.p, counts.data(), counts.size() * sizeof(long long), cudaMemcpyHostToDevice));
        cuda_check(cudaMemsetAsync(sums.p, 0, static_cast<size_t>(k) * d * sizeof(unsigned long long), stream));
        launch_fixed_sums(train, labels.p, m, d, scale, sums.p, stream);
        launch_means(sums.p, dev_counts.p, k, d, inv_scale, centroids, stream);
        cuda_check(cudaGetLastError());
        cuda_check(cudaStreamSynchronize(stream));
        if (std::find(counts.begin(), counts.end(), 0LL) != counts.end()) {
            host_centroids.resize(static_cast<size_t>(k) * d);
            cuda_check(cudaMemcpy(host_centroids.data(), centroids, host_centroids.size() * sizeof(float),
                                  cudaMemcpyDeviceToHost));
            std::vector<double> w(counts.begin(), counts.end());
            split_empty(host_centroids, w, k, d, m, split_rng);
            cuda_check(cudaMemcpy(centroids, host_centroids.data(), host_centroids.size() * sizeof(float),
                                  cudaMemcpyHostToDevice));
        }
    }
}

void ivf_assign(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t *lists, float *dist,
                cudaStream_t stream) {
    require(centroids && x && lists && k > 0 && n > 0 && n <= INT32_MAX && d > 0 && d <= 4096,
            "invalid IVF assignment arguments");
    const int sms = device_sms();
    check_training_input(centroids, k, d, sms);
    check_training_input(x, n, d, sms);
    DeviceBuffer<float> own_dist(dist ? 0 : static_cast<size_t>(n));
    DeviceBuffer<int64_t> wide(static_cast<size_t>(n));
    nearest(centroids, k, x, n, d, dist ? dist : own_dist.p, wide.p, stream);
    launch_narrow_labels(wide.p, n, lists, stream);
    cuda_check(cudaGetLastError());
    cuda_check(cudaStreamSynchronize(stream));
}

VfrIndex *ivf_build(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, int32_t nprobe,
                    const VfrOptions *opt) {
    require(centroids && x && k > 0 && n > 0 && n <= INT32_MAX && d > 0 && d <= 4096, "invalid IVF build arguments");
    const VfrOptions o = resolve_options(opt);
    std::vector<int32_t> lists(static_cast<size_t>(n));
    {
        OwnedStream s;
        DeviceBuffer<int32_t> dev_lists(static_cast<size_t>(n));
        ivf_assign(centroids, k, x, n, d, dev_lists.p, nullptr, s.s);
        cuda_check(cudaMemcpy(lists.data(), dev_lists.p, lists.size() * sizeof(int32_t), cudaMemcpyDeviceToHost));
    }
    // stable counting sort: rows of a list keep their input order, as
    // IndexIVF::add appends them
    std::vector<int32_t> offsets(static_cast<size_t>(k) + 1, 0);
    for (int32_t l : lists) {
        require(l >= 0 && l < k, "IVF list assignment out of range");
        ++offsets[static_cast<size_t>(l) + 1];
    }
    for (int32_t j = 0; j < k; ++j) offsets[j + 1] += offsets[j];
    std::vector<int32_t> cursor(offsets.begin(), offsets.end() - 1);
    std::vector<int64_t> order(static_cast<size_t>(n));
    std::vector<int32_t> ids(static_cast<size_t>(n)), inverse(static_cast<size_t>(n));
    for (int64_t r = 0; r < n; ++r) {
        const int32_t row = cursor[lists[r]]++;
        order[row] = r;
        ids[row] = static_cast<int32_t>(r);
        inverse[r] = row;
    }
    VfrIndex *ix = new_handle(d, k, nprobe, static_cast<size_t>(n), offsets.data(), o);
    try {
        const size_t cbytes = static_cast<size_t>(k) * d * sizeof(float);
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->centroids), cbytes));
        cuda_check(cudaMemcpy(ix->centroids, centroids, cbytes, cudaMemcpyDeviceToDevice));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->offsets), offsets.size() * sizeof(int32_t)));
        cuda_check(cudaMemcpy(ix->offsets, offsets.data(), offsets.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->ids), ids.size() * sizeof(int32_t)));
        cuda_check(cudaMemcpy(ix->ids, ids.data(), ids.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->row_of_id), inverse.size() * sizeof(int32_t)));
        cuda_check(
            cudaMemcpy(ix->row_of_id, inverse.data(), inverse.size() * sizeof(int32_t), cudaMemcpyHostToDevice));
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&ix->vectors), static_cast<size_t>(n) * d * sizeof(float)));
        {
            DeviceBuffer<int64_t> dev_order(order.size());
            cuda_check(cudaMemcpy(dev_order.p, order.data(), order.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
            launch_gather_rows(x, dev_order.p, n, d, ix->vectors, nullptr);
            cuda_check(cudaGetLastError());
            cuda_check(cudaDeviceSynchronize());
        }
        validate_arrays(d, k, nprobe, static_cast<size_t>(n), ix->centroids, static_cast<size_t>(k) * d,
                        offsets.data(), offsets.size(), ix->vectors, static_cast<size_t>(n) * d, ids.data(),
                        ids.size());
        finish_index(ix, o);
    } catch (...) {
        free_index(ix);
        throw;
    }
    return ix;
}

size_t ivf_write(const float *centroids, int32_t k, const float *x, int64_t n, int32_t d, const int32_t *lists,
                 int32_t nprobe, uint8_t *out, size_t capacity) {
    require(centroids && x && lists && k > 0 && n > 0 && d > 0 && d <= 4096 && nprobe > 0 && nprobe <= k,
            "invalid IVF write arguments");
    std::vector<uint64_t> sizes(static_cast<size_t>(k), 0);
    for (int64_t r = 0; r < n; ++r) {
        require(lists[r] >= 0 && lists[r] < k, "IVF list assignment out of range");
        ++sizes[static_cast<size_t>(lists[r])];
    }
    size_t nonempty = 0;
    for (uint64_t s : sizes) nonempty += s > 0;
    const bool full = nonempty > static_cast<size_t>(k) / 2;  // ArrayInvertedLists' directory choice
    const size_t header = 4 + 4 + 8 + 8 + 8 + 1 + 4;
    const size_t total = header + 16 + header + 8 + static_cast<size_t>(k) * d * 4 + 9 + 4 + 16 + 4 + 8 +
                         (full ? static_cast<size_t>(k) * 8 : nonempty * 16) +
                         static_cast<size_t>(n) * (static_cast<size_t>(d) * 4 + 8);
    if (!out || capacity < total) return total;
    uint8_t *p = out;
    auto put = [&](const void *v, size_t bytes) {
        std::memcpy(p, v, bytes);
        p += bytes;
    };
    auto u64 = [&](uint64_t v) { put(&v, 8); };  // little-endian hosts only, like the reader
    auto index_header = [&](const char *kind, int32_t dim, int64_t count) {
        put(kind, 4);
        put(&dim, 4);
        put(&count, 8);
        u64(uint64_t(1) << 20);  // legacy dummy fields, as FAISS writes them
        u64(uint64_t(1) << 20);
        const uint8_t trained = 1;
        put(&trained, 1);
        const int32_t metric = 1;  // METRIC_L2
        put(&metric, 4);
    };
    index_header("IwFl", d, n);
    u64(static_cast<uint64_t>(k));
    u64(static_cast<uint64_t>(nprobe));
    index_header("IxF2", d, k);
    u64(static_cast<uint64_t>(k) * d);
    put(centroids, static_cast<size_t>(k) * d * 4);
    const uint8_t no_map = 0;
    put(&no_map, 1);
    u64(0);
    put("ilar", 4);
    u64(static_cast<uint64_t>(k));
    u64(static_cast<uint64_t>(d) * 4);
    if (full) {
        put("full", 4);
        u64(static_cast<uint64_t>(k));
        for (uint64_t s : sizes) u64(s);
    } else {
        put("sprs", 4);
        u64(2 * nonempty);
        for (int32_t l = 0; l < k; ++l)
            if (sizes[l]) {
                u64(static_cast<uint64_t>(l));
                u64(sizes[l]);
            }
    }
    // per list: the rows in input order, then their ids (the input indices)
    std::vector<int64_t> offsets(static_cast<size_t>(k) + 1, 0);
    for (int32_t l = 0; l < k; ++l) offsets[l + 1] = offsets[l] + static_cast<int64_t>(sizes[l]);
    std::vector<int64_t> cursor(offsets.begin(), offsets.end() - 1), order(static_cast<size_t>(n));
    for (int64_t r = 0; r < n; ++r) order[cursor[lists[r]]++] = r;
    for (int32_t l = 0; l < k; ++l) {
        for (int64_t i = offsets[l]; i < offsets[l + 1]; ++i) put(x + order[i] * d, static_cast<size_t>(d) * 4);
        for (int64_t i = offsets[l]; i < offsets[l + 1]; ++i) u64(static_cast<uint64_t>(order[i]));
    }
    return total;
}

}  // namespace vfr
