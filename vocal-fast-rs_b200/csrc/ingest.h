// Host -> device ingest of index payloads: a staged, multi-threaded upload
// through pinned buffers and the content hash that keys shared storage.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace vfr {

// One contiguous piece of the source image and where it lands in the device
// buffer (byte offsets).
struct UploadSpan {
    const uint8_t *src;
    size_t bytes;
    size_t dst;
};

// Copies every span to dst + span.dst on `device` and returns when all copies
// are complete.  Large payloads are split across host threads, each copying
// 8 MiB pieces into its own pair of pinned buffers while the previous piece
// is in flight on its own stream (the pageable path of cudaMemcpy runs at a
// fifth of the pinned DMA rate).
void staged_upload(void *dst, const std::vector<UploadSpan> &spans, int device);

// 128-bit content hash of `length` bytes, independent of the thread count:
// 1 MiB blocks hashed in parallel, then the block digests in order.
struct ContentHash {
    uint64_t lo = 0, hi = 0;
    bool operator<(const ContentHash &o) const { return lo != o.lo ? lo < o.lo : hi < o.hi; }
    bool operator==(const ContentHash &o) const { return lo == o.lo && hi == o.hi; }
};
ContentHash content_hash(const uint8_t *bytes, size_t length);

// A read-only mapping of a whole file (unmapped on destruction); rows are
// read from it by the upload threads, so the page cache is the only host
// copy.
struct MappedFile {
    const uint8_t *data = nullptr;
    size_t size = 0;
    explicit MappedFile(const char *path);
    ~MappedFile();
    MappedFile(const MappedFile &) = delete;
    MappedFile &operator=(const MappedFile &) = delete;
};

}  // namespace vfr
