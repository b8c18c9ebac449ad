// Host side of the index ingest: staged upload and content hash.
//
// The reference uploads each array with one pageable cudaMemcpy
// (crates/vocal-tensorrt/native/retrieval.cu:66-87); from pageable memory the
// driver stages through its own small pinned buffer on one thread, about
// 10 GB/s here, so a 12 GB index takes over a second.  staged_upload splits
// the payload across host threads; each copies 8 MiB pieces into its own two
// pinned buffers and issues the DMA of one piece on its own stream while it
// copies the next, which keeps the copy engines near the pinned rate.
#include "ingest.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>

namespace vfr {
namespace {

constexpr size_t kPiece = size_t(8) << 20;
constexpr size_t kHashBlock = size_t(1) << 20;

int host_threads(size_t work_units) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t t = std::min<size_t>({static_cast<size_t>(hw), size_t(16), std::max<size_t>(work_units, 1)});
    return static_cast<int>(t);
}

void check(cudaError_t rc, const char *what) {
    if (rc != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(rc));
}

// One worker's stream, events and pinned pair; released on every path.
struct Stage {
    cudaStream_t stream = nullptr;
    cudaEvent_t done[2] = {nullptr, nullptr};
    void *pinned[2] = {nullptr, nullptr};
    bool busy[2] = {false, false};
    // not in the constructor, so the destructor releases a partial setup
    void init(int device) {
        check(cudaSetDevice(device), "cudaSetDevice");
        check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
        for (int k = 0; k < 2; ++k) {
            check(cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming), "cudaEventCreate");
            check(cudaHostAlloc(&pinned[k], kPiece, cudaHostAllocDefault), "cudaHostAlloc staging buffer");
        }
    }
    ~Stage() {
        if (stream) cudaStreamSynchronize(stream);
        for (int k = 0; k < 2; ++k) {
            if (pinned[k]) cudaFreeHost(pinned[k]);
            if (done[k]) cudaEventDestroy(done[k]);
        }
        if (stream) cudaStreamDestroy(stream);
    }
    void put(uint8_t *dst, const uint8_t *src, size_t bytes, int slot) {
        if (busy[slot]) check(cudaEventSynchronize(done[slot]), "staging wait");
        std::memcpy(pinned[slot], src, bytes);
        check(cudaMemcpyAsync(dst, pinned[slot], bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync");
        check(cudaEventRecord(done[slot], stream), "cudaEventRecord");
        busy[slot] = true;
    }
};

// XXH64's round and avalanche (Y. Collet, xxHash specification), four lanes
// over 32-byte stripes; the tail is zero-padded into a last stripe and the
// length folded into both finalisations.
constexpr uint64_t kP1 = 0x9E3779B185EBCA87ull, kP2 = 0xC2B2AE3D27D4EB4Full, kP3 = 0x165667B19E3779F9ull,
                   kP4 = 0x85EBCA77C2B2AE63ull, kP5 = 0x27D4EB2F165667C5ull;

inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
inline uint64_t round64(uint64_t acc, uint64_t in) { return rotl(acc + in * kP2, 31) * kP1; }
inline uint64_t avalanche(uint64_t h) {
    h ^= h >> 33;
    h *= kP2;
    h ^= h >> 29;
    h *= kP3;
    h ^= h >> 32;
    return h;
}

ContentHash hash_block(const uint8_t *p, size_t n, uint64_t seed) {
    uint64_t a[4] = {seed + kP1 + kP2, seed + kP2, seed, seed - kP1};
    size_t i = 0;
    for (; i + 32 <= n; i += 32) {
        uint64_t w[4];
        std::memcpy(w, p + i, 32);
        for (int k = 0; k < 4; ++k) a[k] = round64(a[k], w[k]);
    }
    if (i < n) {
        uint64_t w[4] = {0, 0, 0, 0};
        std::memcpy(w, p + i, n - i);
        for (int k = 0; k < 4; ++k) a[k] = round64(a[k], w[k]);
    }
    uint64_t h = rotl(a[0], 1) + rotl(a[1], 7) + rotl(a[2], 12) + rotl(a[3], 18);
    uint64_t g = rotl(a[3], 3) ^ rotl(a[2], 17) ^ rotl(a[1], 29) ^ rotl(a[0], 41);
    for (int k = 0; k < 4; ++k) {
        h = (h ^ round64(0, a[k])) * kP1 + kP4;
        g = (g ^ round64(kP5, a[3 - k])) * kP3 + kP2;
    }
    return {avalanche(h ^ static_cast<uint64_t>(n)), avalanche(g + static_cast<uint64_t>(n) * kP5)};
}

}  // namespace

void staged_upload(void *dst, const std::vector<UploadSpan> &spans, int device) {
    size_t total = 0;
    for (const auto &s : spans) total += s.bytes;
    if (total == 0) return;
    auto *base = static_cast<uint8_t *>(dst);
    check(cudaSetDevice(device), "cudaSetDevice");
    if (total <= 4 * kPiece) {
        for (const auto &s : spans)
            if (s.bytes) check(cudaMemcpy(base + s.dst, s.src, s.bytes, cudaMemcpyHostToDevice), "cudaMemcpy");
        return;
    }
    const int workers = host_threads(total / (4 * kPiece));
    std::mutex failure_lock;
    std::string failure;
    std::atomic<bool> stop{false};
    auto work = [&](int w) {
        try {
            Stage stage;
            stage.init(device);
            // this worker's share of the concatenated spans, in 4 KiB units
            const size_t lo = total / 4096 * w / workers * 4096;
            const size_t hi = w + 1 == workers ? total : total / 4096 * (w + 1) / workers * 4096;
            size_t at = 0;
            int slot = 0;
            for (const auto &s : spans) {
                const size_t a = std::max(lo, at), b = std::min(hi, at + s.bytes);
                for (size_t x = a; x < b && !stop.load(std::memory_order_relaxed); x += kPiece) {
                    const size_t len = std::min(kPiece, b - x);
                    stage.put(base + s.dst + (x - at), s.src + (x - at), len, slot);
                    slot ^= 1;
                }
                at += s.bytes;
            }
            check(cudaStreamSynchronize(stage.stream), "staged upload");
        } catch (const std::exception &e) {
            stop = true;
            std::lock_guard<std::mutex> g(failure_lock);
            if (failure.empty()) failure = e.what();
        }
    };
    std::vector<std::thread> pool;
    for (int w = 1; w < workers; ++w) pool.emplace_back(work, w);
    work(0);
    for (auto &t : pool) t.join();
    check(cudaSetDevice(device), "cudaSetDevice");
    if (!failure.empty()) throw std::runtime_error(failure);
}

ContentHash content_hash(const uint8_t *bytes, size_t length) {
    const size_t blocks = (length + kHashBlock - 1) / kHashBlock;
    std::vector<ContentHash> digest(std::max<size_t>(blocks, 1));
    std::atomic<size_t> next{0};
    auto work = [&] {
        for (size_t b = next++; b < blocks; b = next++) {
            const size_t off = b * kHashBlock;
            digest[b] = hash_block(bytes + off, std::min(kHashBlock, length - off), b);
        }
    };
    const int workers = host_threads(blocks / 8);
    std::vector<std::thread> pool;
    for (int w = 1; w < workers; ++w) pool.emplace_back(work);
    work();
    for (auto &t : pool) t.join();
    ContentHash h = hash_block(reinterpret_cast<const uint8_t *>(digest.data()), digest.size() * sizeof(ContentHash),
                               static_cast<uint64_t>(length));
    return h;
}

MappedFile::MappedFile(const char *path) {
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw std::runtime_error(std::string("cannot open retrieval index file ") + path + ": " + std::strerror(errno));
    struct stat st {};
    if (::fstat(fd, &st) != 0) {
        const int e = errno;
        ::close(fd);
        throw std::runtime_error(std::string("cannot stat retrieval index file ") + path + ": " + std::strerror(e));
    }
    size = static_cast<size_t>(st.st_size);
    if (size > 0) {
        void *p = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            const int e = errno;
            ::close(fd);
            throw std::runtime_error(std::string("cannot map retrieval index file ") + path + ": " + std::strerror(e));
        }
        ::madvise(p, size, MADV_WILLNEED);
        data = static_cast<const uint8_t *>(p);
    }
    ::close(fd);
}

MappedFile::~MappedFile() {
    if (data) ::munmap(const_cast<uint8_t *>(data), size);
}

}  // namespace vfr
