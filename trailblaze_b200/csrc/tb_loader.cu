// tb_loader.cu — model upload into one device arena, streamed through pinned
// staging, with per-rank shard extraction at load time.
//
// Replaces the load path of layer4/tb_gguf.c:469-520 (tb_gguf_cuda_upload_all)
// and layer4/tb_gguf_dequant.cu:411-416 (tb_cuda_upload_tensor): there every
// tensor is one cudaMalloc plus one synchronous cudaMemcpy from the mmap'd
// file, i.e. from pageable memory, which the driver stages through its own
// small pinned buffer one piece at a time.  Here:
//   * one cudaMalloc for the whole model (an arena); tensors are 256-byte
//     aligned sub-ranges, so a model's weights are one allocation to map,
//     shard and free;
//   * the host bytes are copied in chunks into two pinned staging buffers on
//     the host while the previous chunk's DMA runs (cudaMemcpyAsync from
//     pinned memory on the arena's stream, one event per buffer), so the host
//     copy and the PCIe / NVLink-C2C transfer overlap;
//   * a tensor-parallel rank can take its shard directly: a row range (q/k/v
//     heads, FFN row pairs, vocabulary rows: a contiguous byte range of the
//     GGUF tensor) or a column range (o / down K slices: the same block range
//     of every row, gathered on the host into the staging buffer), so no rank
//     ever holds the whole tensor on its device.
// Uploads are blocking and return the device pointer; the raw GGUF bytes are
// not changed (the kernels read the file's block layout as it is).
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/tb_gguf_dequant.h"
#include "tb_common.cuh"
#include "tb_internal.h"

namespace {

constexpr size_t kChunk = 32u << 20;   // bytes per staging buffer
constexpr size_t kAlign = 256;

struct Arena {
    uint8_t *base = nullptr;
    size_t cap = 0, used = 0;
    int dev = 0;
    cudaStream_t st = nullptr;
    uint8_t *pin[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    std::mutex mu;
};

bool ok(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    fprintf(stderr, "[tb_cuda] arena: %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

void arena_free(Arena *a)
{
    if (!a) return;
    if (a->st) cudaStreamSynchronize(a->st);
    for (int i = 0; i < 2; ++i) {
        if (a->pin[i]) cudaFreeHost(a->pin[i]);
        if (a->done[i]) cudaEventDestroy(a->done[i]);
    }
    if (a->st) cudaStreamDestroy(a->st);
    if (a->base) cudaFree(a->base);
    delete a;
}

// Reserves n bytes (256-byte aligned start); nullptr when the arena is full.
uint8_t *reserve(Arena *a, size_t n)
{
    const size_t off = (a->used + kAlign - 1) & ~(kAlign - 1);
    if (off > a->cap || n > a->cap - off) {
        fprintf(stderr, "[tb_cuda] arena: %zu bytes do not fit (%zu of %zu used)\n", n, a->used, a->cap);
        return nullptr;
    }
    a->used = off + n;
    return a->base + off;
}

// Streams `total` bytes to dst: fill(chunk_dst_host, offset, bytes) writes the
// host bytes of [offset, offset + bytes) into pinned memory.  Two staging
// buffers alternate: the host fills one while the other's copy runs.
template <class Fill>
bool stream_up(Arena *a, uint8_t *dst, size_t total, Fill fill)
{
    size_t off = 0;
    int b = 0;
    while (off < total) {
        const size_t n = total - off < kChunk ? total - off : kChunk;
        if (!ok(cudaEventSynchronize(a->done[b]), "staging wait")) return false;   // its previous copy is done
        fill(a->pin[b], off, n);
        if (!ok(cudaMemcpyAsync(dst + off, a->pin[b], n, cudaMemcpyHostToDevice, a->st), "copy") ||
            !ok(cudaEventRecord(a->done[b], a->st), "event"))
            return false;
        off += n;
        b ^= 1;
    }
    return ok(cudaStreamSynchronize(a->st), "sync");
}

}  // namespace

extern "C" {

void *tb_cuda_arena_create(size_t bytes)
{
    if (bytes == 0) return nullptr;
    Arena *a = new Arena;
    cudaGetDevice(&a->dev);
    a->cap = bytes;
    bool good = ok(cudaMalloc(&a->base, bytes), "alloc") &&
                ok(cudaStreamCreateWithFlags(&a->st, cudaStreamNonBlocking), "stream");
    for (int i = 0; good && i < 2; ++i)
        good = ok(cudaMallocHost(&a->pin[i], kChunk), "pinned staging") &&
               ok(cudaEventCreateWithFlags(&a->done[i], cudaEventDisableTiming), "event") &&
               ok(cudaEventRecord(a->done[i], a->st), "event");
    if (!good) {
        arena_free(a);
        return nullptr;
    }
    return a;
}

void *tb_cuda_arena_upload(void *arena, const void *host, size_t n)
{
    Arena *a = static_cast<Arena *>(arena);
    if (!a || !host || n == 0) return nullptr;
    const tb::NvtxRange nvtx("tb.arena.upload");
    std::lock_guard<std::mutex> lk(a->mu);
    uint8_t *dst = reserve(a, n);
    if (!dst) return nullptr;
    const uint8_t *src = static_cast<const uint8_t *>(host);
    if (!stream_up(a, dst, n, [&](uint8_t *pin, size_t off, size_t len) { memcpy(pin, src + off, len); }))
        return nullptr;
    return dst;
}

void *tb_cuda_arena_upload_rows(void *arena, const void *host, size_t row_bytes, int r_lo, int r_hi)
{
    if (!host || row_bytes == 0 || r_lo < 0 || r_hi <= r_lo) return nullptr;
    return tb_cuda_arena_upload(arena, static_cast<const uint8_t *>(host) + row_bytes * static_cast<size_t>(r_lo),
                                row_bytes * static_cast<size_t>(r_hi - r_lo));
}

void *tb_cuda_arena_upload_cols(void *arena, const void *host, int M, size_t row_bytes, size_t b_lo, size_t b_hi)
{
    Arena *a = static_cast<Arena *>(arena);
    if (!a || !host || M <= 0 || b_hi <= b_lo || b_hi > row_bytes) return nullptr;
    const size_t w = b_hi - b_lo;
    if (w > kChunk) {
        fprintf(stderr, "[tb_cuda] arena: a column slice of %zu bytes per row exceeds the staging buffer\n", w);
        return nullptr;
    }
    const tb::NvtxRange nvtx("tb.arena.upload_cols");
    std::lock_guard<std::mutex> lk(a->mu);
    uint8_t *dst = reserve(a, w * static_cast<size_t>(M));
    if (!dst) return nullptr;
    const uint8_t *src = static_cast<const uint8_t *>(host);
    // chunks of whole rows: the staging buffer holds kChunk / w slice rows
    const size_t rows_per = kChunk / w;
    size_t done = 0;
    int b = 0;
    while (done < static_cast<size_t>(M)) {
        const size_t nr = static_cast<size_t>(M) - done < rows_per ? static_cast<size_t>(M) - done : rows_per;
        if (!ok(cudaEventSynchronize(a->done[b]), "staging wait")) return nullptr;
        for (size_t r = 0; r < nr; ++r) memcpy(a->pin[b] + r * w, src + (done + r) * row_bytes + b_lo, w);
        if (!ok(cudaMemcpyAsync(dst + done * w, a->pin[b], nr * w, cudaMemcpyHostToDevice, a->st), "copy") ||
            !ok(cudaEventRecord(a->done[b], a->st), "event"))
            return nullptr;
        done += nr;
        b ^= 1;
    }
    return ok(cudaStreamSynchronize(a->st), "sync") ? dst : nullptr;
}

size_t tb_cuda_arena_used(void *arena)
{
    Arena *a = static_cast<Arena *>(arena);
    if (!a) return 0;
    std::lock_guard<std::mutex> lk(a->mu);
    return a->used;
}

void tb_cuda_arena_destroy(void *arena) { arena_free(static_cast<Arena *>(arena)); }

}  // extern "C"
