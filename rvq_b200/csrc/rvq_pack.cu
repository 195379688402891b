// Native loader of an artifact pack: the compressor's torch.save artifact
// (compress_full_model.py:624-631) rewritten once as a flat file -- a JSON
// header followed by every tensor's raw bytes, page aligned -- so that loading
// it (infer_compressed_layerwise_triton.py:421-432: torch.load, then one
// .to(device) per tensor) becomes a single streamed host-to-device copy into
// one device buffer, with no unpickling and no per-tensor transfers.
//
// The data region is read with pread() by a reader thread into a ring of
// pinned host buffers while the calling thread issues one cudaMemcpyAsync per
// filled buffer on the caller's stream; a CUDA event per buffer tells the
// reader when it may refill it.  File reads and DMA overlap.

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

constexpr size_t kBufBytes = 32u << 20;      // one pinned staging buffer
constexpr int kBufs = 3;

struct Ring {
    std::mutex mu;
    std::condition_variable cv;
    size_t filled[kBufs] = {0, 0, 0};        // bytes ready in buffer i (0: empty)
    bool ready[kBufs] = {false, false, false};
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
    void* host[kBufs] = {nullptr, nullptr, nullptr};
    cudaEvent_t done[kBufs] = {nullptr, nullptr, nullptr};
    int rc = RVQ_OK;
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
        const uint64_t nchunks = (nbytes + kBufBytes - 1) / kBufBytes;
        // reader: chunk c goes to buffer c % kBufs once the copy of chunk c - kBufs is done
        std::thread reader([&]() {
            for (uint64_t c = 0; c < nchunks; ++c) {
                const int b = (int)(c % kBufs);
                {
                    std::unique_lock<std::mutex> lk(ring.mu);
                    ring.cv.wait(lk, [&] { return !ring.ready[b] || ring.failed; });
                    if (ring.failed) return;
                }
                if (c >= (uint64_t)kBufs) {
                    const cudaError_t e = cudaEventSynchronize(done[b]);
                    if (e != cudaSuccess) {
                        std::lock_guard<std::mutex> lk(ring.mu);
                        ring.failed = true;
                        ring.err = RVQ_ERR_CUDA;
                        last_cuda_error_slot() = (int)e;
                        ring.cv.notify_all();
                        return;
                    }
                }
                const uint64_t begin = c * kBufBytes;
                const size_t len = (size_t)((nbytes - begin) < kBufBytes ? (nbytes - begin) : kBufBytes);
                size_t got = 0;
                while (got < len) {
                    const ssize_t r = pread(fd, (char*)host[b] + got, len - got, (off_t)(offset + begin + got));
                    if (r < 0 && errno == EINTR) continue;
                    if (r <= 0) {
                        std::lock_guard<std::mutex> lk(ring.mu);
                        ring.failed = true;
                        ring.err = RVQ_ERR_INVALID;
                        ring.cv.notify_all();
                        return;
                    }
                    got += (size_t)r;
                }
                std::lock_guard<std::mutex> lk(ring.mu);
                ring.filled[b] = len;
                ring.ready[b] = true;
                ring.cv.notify_all();
            }
        });
        for (uint64_t c = 0; c < nchunks; ++c) {
            const int b = (int)(c % kBufs);
            size_t len = 0;
            {
                std::unique_lock<std::mutex> lk(ring.mu);
                ring.cv.wait(lk, [&] { return ring.ready[b] || ring.failed; });
                if (ring.failed) {
                    rc = ring.err;
                    break;
                }
                len = ring.filled[b];
            }
            cudaError_t e = cudaMemcpyAsync((char*)dst + c * kBufBytes, host[b], len, cudaMemcpyHostToDevice, stream);
            if (e == cudaSuccess) e = cudaEventRecord(done[b], stream);
            std::lock_guard<std::mutex> lk(ring.mu);
            if (e != cudaSuccess) {
                last_cuda_error_slot() = (int)e;
                rc = RVQ_ERR_CUDA;
                ring.failed = true;
                ring.cv.notify_all();
                break;
            }
            ring.ready[b] = false;            // the reader refills it after done[b]
            ring.cv.notify_all();
        }
        reader.join();
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
