// Native loader of an artifact pack: the compressor's torch.save artifact
// (compress_full_model.py:624-631) rewritten once as a flat file -- a JSON
// header followed by every tensor's raw bytes, page aligned -- so that loading
// it (infer_compressed_layerwise_triton.py:421-432: torch.load, then one
// .to(device) per tensor) becomes a single streamed host-to-device copy into
// one device buffer, with no unpickling and no per-tensor transfers.
//
// The data region is read with pread() by four reader threads into a ring of
// pinned host buffers while the calling thread issues one cudaMemcpyAsync per
// filled buffer, in file order, on the caller's stream; a CUDA event per
// buffer tells its reader when it may refill it.  File reads (page-cache
// copies or disk) run in parallel and overlap the DMA.

#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

#include "rvq_b200.h"
#include "rvq_common.cuh"

namespace rvq {
namespace pack {

constexpr size_t kBufBytes = 16u << 20;      // one pinned staging buffer
constexpr int kReaders = 4;                  // pread threads
constexpr int kBufs = 2 * kReaders;          // ring: each reader owns buffers r and r + kReaders

struct Ring {
    std::mutex mu;
    std::condition_variable cv;
    int64_t holds[kBufs];                    // chunk whose bytes buffer b holds (-1: none)
    int64_t copied = -1;                     // highest chunk whose copy has been issued
    size_t len[kBufs];
    bool failed = false;
    int err = 0;
};

int load(const char* path, uint64_t offset, uint64_t nbytes, void* dst, cudaStream_t stream) {
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return RVQ_ERR_INVALID;
    struct stat st;
    if (fstat(fd, &st) != 0 || (uint64_t)st.st_size < offset + nbytes) {
        close(fd);
        return RVQ_ERR_INVALID;
    }
    posix_fadvise(fd, (off_t)offset, (off_t)nbytes, POSIX_FADV_SEQUENTIAL);
    void* host[kBufs] = {};
    cudaEvent_t done[kBufs] = {};
    int rc = RVQ_OK;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) rc = RVQ_ERR_UNAVAILABLE;
    for (int i = 0; i < kBufs && rc == RVQ_OK; ++i) {
        cudaError_t e = cudaHostAlloc(&host[i], kBufBytes, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
        if (e != cudaSuccess) {
            last_cuda_error_slot() = (int)e;
            rc = RVQ_ERR_CUDA;
        }
    }
    if (rc == RVQ_OK && nbytes > 0) {
        Ring ring;
        for (int b = 0; b < kBufs; ++b) ring.holds[b] = -1;
        const int64_t nchunks = (int64_t)((nbytes + kBufBytes - 1) / kBufBytes);
        auto fail = [&](int code) {
            std::lock_guard<std::mutex> lk(ring.mu);
            ring.failed = true;
            ring.err = code;
            ring.cv.notify_all();
        };
        // reader r reads chunks r, r + kReaders, ...; chunk c goes to buffer c % kBufs once
        // the copy of chunk c - kBufs (the buffer's previous content) has been issued and finished
        std::vector<std::thread> readers;
        for (int r = 0; r < kReaders; ++r) {
            readers.emplace_back([&, r]() {
                cudaSetDevice(device);               // the events belong to the caller's device
                for (int64_t c = r; c < nchunks; c += kReaders) {
                    const int b = (int)(c % kBufs);
                    {
                        std::unique_lock<std::mutex> lk(ring.mu);
                        ring.cv.wait(lk, [&] { return ring.failed || ring.copied >= c - kBufs; });
                        if (ring.failed) return;
                    }
                    if (c >= kBufs) {
                        const cudaError_t e = cudaEventSynchronize(done[b]);
                        if (e != cudaSuccess) {
                            last_cuda_error_slot() = (int)e;
                            fail(RVQ_ERR_CUDA);
                            return;
                        }
                    }
                    const uint64_t begin = (uint64_t)c * kBufBytes;
                    const size_t len = (size_t)((nbytes - begin) < kBufBytes ? (nbytes - begin) : kBufBytes);
                    size_t got = 0;
                    while (got < len) {
                        const ssize_t n = pread(fd, (char*)host[b] + got, len - got, (off_t)(offset + begin + got));
                        if (n < 0 && errno == EINTR) continue;
                        if (n <= 0) {
                            fail(RVQ_ERR_INVALID);
                            return;
                        }
                        got += (size_t)n;
                    }
                    std::lock_guard<std::mutex> lk(ring.mu);
                    ring.len[b] = len;
                    ring.holds[b] = c;
                    ring.cv.notify_all();
                }
            });
        }
        // copies in chunk order, each as soon as its buffer is filled
        for (int64_t c = 0; c < nchunks; ++c) {
            const int b = (int)(c % kBufs);
            size_t len = 0;
            {
                std::unique_lock<std::mutex> lk(ring.mu);
                ring.cv.wait(lk, [&] { return ring.failed || ring.holds[b] == c; });
                if (ring.failed) {
                    rc = ring.err;
                    break;
                }
                len = ring.len[b];
            }
            cudaError_t e = cudaMemcpyAsync((char*)dst + (uint64_t)c * kBufBytes, host[b], len,
                                            cudaMemcpyHostToDevice, stream);
            if (e == cudaSuccess) e = cudaEventRecord(done[b], stream);
            if (e != cudaSuccess) {
                last_cuda_error_slot() = (int)e;
                rc = RVQ_ERR_CUDA;
                fail(RVQ_ERR_CUDA);
                break;
            }
            std::lock_guard<std::mutex> lk(ring.mu);
            ring.copied = c;
            ring.cv.notify_all();
        }
        for (auto& t : readers) t.join();
        if (rc == RVQ_OK && ring.failed) rc = ring.err;
    }
    // the pinned buffers are freed only after their copies have finished
    for (int i = 0; i < kBufs; ++i) {
        if (done[i]) {
            cudaEventSynchronize(done[i]);
            cudaEventDestroy(done[i]);
        }
    }
    for (int i = 0; i < kBufs; ++i)
        if (host[i]) cudaFreeHost(host[i]);
    close(fd);
    return rc;
}

}  // namespace pack
}  // namespace rvq

extern "C" int rvq_pack_load(const char* path, uint64_t offset, uint64_t nbytes, void* device_dst, void* stream) {
    if (path == nullptr || (nbytes > 0 && device_dst == nullptr)) return RVQ_ERR_INVALID;
    return rvq::pack::load(path, offset, nbytes, device_dst, (cudaStream_t)stream);
}
