// Peer groups: a one-kernel all-gather of output-row shards over NVLink.
//
// One process per GPU. Each rank's group owns one cudaMalloc allocation:
//   [0, 8)      arrival counter (u64): signals received from peers, one per pushing CTA
//   [8, 16)     expected count (u64): advanced by each wait
//   [256, ...)  the output buffer handed to callers (`bytes` long), identical layout on every rank
// The ranks exchange CUDA IPC handles of these allocations and map each other's. The all-gather
// kernel (a fixed grid of AG_CTAS CTAs on every rank) copies this rank's chunks of the buffer to
// the same offsets in every peer's buffer with coalesced 16-byte stores over NVLink (plain
// stores; no multicast). Each CTA then passes a CTA barrier, fences at system scope and adds 1
// to every peer's arrival counter with release semantics; CTA 0 advances this rank's expected
// count by (world - 1) * AG_CTAS and spins, with an acquire load and a 2 s bound, until the
// arrivals reach it. Both counts live on the device, so a captured CUDA graph stays correct
// across replays.
#include <cstring>

#include "jkb_internal.h"

struct jkb_peer_group {
    uint32_t magic;
    int world, rank;
    size_t bytes;
    uint8_t *base;  // local allocation
    uint8_t *peer_base[JKB_PEER_MAX_RANKS];  // mapped allocations (peer_base[rank] == base)
    bool opened;
    cudaIpcMemHandle_t handle;
    int device;
};

namespace jkb {

constexpr uint32_t PEER_MAGIC = 0x4A4B5031u;  // "JKP1"
constexpr size_t PEER_HDR = 256;              // counters and padding
constexpr unsigned long long PEER_WAIT_NS = 2000000000ull;
constexpr int AG_CTAS = 16;                   // CTAs of every rank's all-gather launch
constexpr int AG_THREADS = 256;

static bool check_pg(const jkb_peer_group *pg) { return pg && pg->magic == PEER_MAGIC; }

namespace {

struct AgArgs {
    int world, rank, nchunk;
    unsigned long long off[JKB_PEER_MAX_CHUNKS], len[JKB_PEER_MAX_CHUNKS];  // bytes
    uint8_t *data[JKB_PEER_MAX_RANKS];                 // every rank's buffer (data region)
    unsigned long long *cnt[JKB_PEER_MAX_RANKS];       // every rank's arrival counter
    unsigned long long *expected;                      // this rank's expected count
    unsigned long long arrivals;                       // added to it by this launch's wait
    int *err;
};

// Spins (thread 0 of the calling CTA) until *cnt >= (*expected += add); bounded by PEER_WAIT_NS.
__device__ void bounded_arrival_wait(unsigned long long *cnt, unsigned long long *expected,
                                     unsigned long long add, int *err) {
    const unsigned long long target = *expected + add;
    *expected = target;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (uint32_t i = 0;; i++) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(cnt) : "memory");
        if (v >= target) return;
        if ((i & 63) == 63) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > PEER_WAIT_NS) {
                atomicOr(err, 2);
                return;
            }
        }
        __nanosleep(64);
    }
}

__global__ void __launch_bounds__(AG_THREADS) peer_allgather_kernel(AgArgs a) {
    // Launched as a programmatic dependent of the kernel before it (the step's last GEMV): wait
    // for that grid's rows, then let the next step's first kernel launch and load its weights
    // while this one pushes rows and waits for the peers' (its activations wait for this grid).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" :::);
    const uint8_t *src = a.data[a.rank];
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t nthr = (size_t)gridDim.x * blockDim.x;
    for (int c = 0; c < a.nchunk; c++) {
        const size_t off = a.off[c], len = a.len[c];
        // 4-byte head up to a 16-byte boundary, 16-byte body, 4-byte tail
        const size_t head = ((16 - (off & 15)) & 15) < len ? ((16 - (off & 15)) & 15) : len;
        const size_t body = (len - head) & ~(size_t)15;
        for (size_t i = tid; i < (body >> 4); i += nthr) {
            const size_t o = off + head + (i << 4);
            const uint4 v = *reinterpret_cast<const uint4 *>(src + o);
            for (int p = 0; p < a.world; p++)
                if (p != a.rank) *reinterpret_cast<uint4 *>(a.data[p] + o) = v;
        }
        const size_t tail = len - head - body;
        for (size_t i = tid; i < ((head + tail) >> 2); i += nthr) {
            const size_t o = i < (head >> 2) ? off + (i << 2) : off + head + body + ((i - (head >> 2)) << 2);
            const uint32_t v = *reinterpret_cast<const uint32_t *>(src + o);
            for (int p = 0; p < a.world; p++)
                if (p != a.rank) *reinterpret_cast<uint32_t *>(a.data[p] + o) = v;
        }
    }
    // The CTA barrier orders every thread's stores before thread 0's system-scope fence and
    // release, which are cumulative over them; the peer's acquire in its wait sees the data.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < a.world; p++)
            if (p != a.rank)
                asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(a.cnt[p]) : "memory");
        if (blockIdx.x == 0)
            bounded_arrival_wait(a.cnt[a.rank], a.expected, a.arrivals, a.err);
    }
}

__global__ void peer_wait_kernel(unsigned long long *cnt, unsigned long long *expected,
                                 unsigned long long arrivals, int *err) {
    if (threadIdx.x == 0) bounded_arrival_wait(cnt, expected, arrivals, err);
}

}  // namespace
}  // namespace jkb

using namespace jkb;

extern "C" {

int jkb_peer_group_create(int world, int rank, size_t bytes, jkb_peer_group **out) {
    static const char *fn = "peer_group_create";
    if (!out) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null out");
    *out = nullptr;
    if (world < 1 || world > JKB_PEER_MAX_RANKS || rank < 0 || rank >= world)
        return fail(JKB_E_BOUNDS, fn, 0, (size_t)rank, (size_t)world,
                    "rank %d of world %d (1..%d ranks)", rank, world, JKB_PEER_MAX_RANKS);
    if (bytes == 0 || bytes % 16)
        return fail(JKB_E_BOUNDS, fn, 0, bytes, 0, "buffer bytes %zu (non-zero multiple of 16)",
                    bytes);
    jkb_peer_group *pg = new jkb_peer_group();
    memset(pg, 0, sizeof(*pg));
    pg->world = world;
    pg->rank = rank;
    pg->bytes = bytes;
    cudaError_t e = cudaGetDevice(&pg->device);
    if (e == cudaSuccess) e = cudaMalloc(&pg->base, PEER_HDR + bytes);
    if (e == cudaSuccess) e = cudaMemset(pg->base, 0, PEER_HDR + bytes);
    if (e == cudaSuccess && world > 1) e = cudaIpcGetMemHandle(&pg->handle, pg->base);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (pg->base) cudaFree(pg->base);
        delete pg;
        return fail_cuda(e, "jkb_peer_group_create");
    }
    pg->peer_base[rank] = pg->base;
    pg->opened = world == 1;
    pg->magic = PEER_MAGIC;
    *out = pg;
    return JKB_OK;
}

int jkb_peer_group_handle(const jkb_peer_group *pg, void *handle) {
    if (!check_pg(pg) || !handle)
        return fail(JKB_E_INVALID, "peer_group_handle", 0, 0, 0, "null group or handle");
    static_assert(sizeof(cudaIpcMemHandle_t) == JKB_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &pg->handle, JKB_PEER_HANDLE_BYTES);
    return JKB_OK;
}

int jkb_peer_group_open(jkb_peer_group *pg, const void *handles) {
    static const char *fn = "peer_group_open";
    if (!check_pg(pg) || !handles) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null group or handles");
    if (pg->opened) return JKB_OK;
    const uint8_t *h = static_cast<const uint8_t *>(handles);
    for (int p = 0; p < pg->world; p++) {
        if (p == pg->rank) continue;
        cudaIpcMemHandle_t ih;
        memcpy(&ih, h + (size_t)p * JKB_PEER_HANDLE_BYTES, JKB_PEER_HANDLE_BYTES);
        void *ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, ih, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; q++)
                if (q != pg->rank && pg->peer_base[q]) {
                    cudaIpcCloseMemHandle(pg->peer_base[q]);
                    pg->peer_base[q] = nullptr;
                }
            return fail_cuda(e, "jkb_peer_group_open (cudaIpcOpenMemHandle)");
        }
        pg->peer_base[p] = static_cast<uint8_t *>(ptr);
    }
    pg->opened = true;
    return JKB_OK;
}

int jkb_peer_group_buffer(const jkb_peer_group *pg, void **local, size_t *bytes) {
    if (!check_pg(pg)) return fail(JKB_E_INVALID, "peer_group_buffer", 0, 0, 0, "null group");
    if (local) *local = pg->base + PEER_HDR;
    if (bytes) *bytes = pg->bytes;
    return JKB_OK;
}

int jkb_peer_group_allgather(jkb_peer_group *pg, const size_t *offset, const size_t *len,
                             size_t n, void *stream) {
    static const char *fn = "peer_group_allgather";
    if (!check_pg(pg)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed group");
    if (!pg->opened) return fail(JKB_E_INVALID, fn, 0, 0, 0, "peer group not opened");
    if (n > JKB_PEER_MAX_CHUNKS || (n && (!offset || !len)))
        return fail(JKB_E_BOUNDS, fn, 0, n, JKB_PEER_MAX_CHUNKS, "%zu chunks (limit %d)", n,
                    JKB_PEER_MAX_CHUNKS);
    AgArgs a = {};
    a.world = pg->world;
    a.rank = pg->rank;
    a.nchunk = (int)n;
    for (size_t i = 0; i < n; i++) {
        if (offset[i] % 4 || len[i] % 4 || offset[i] > pg->bytes || len[i] > pg->bytes - offset[i])
            return fail(JKB_E_BOUNDS, fn, offset[i], len[i], pg->bytes,
                        "chunk %zu [%zu, +%zu) not 4-byte aligned or outside the %zu-byte buffer",
                        i, offset[i], len[i], pg->bytes);
        a.off[i] = offset[i];
        a.len[i] = len[i];
    }
    if (pg->world == 1) return JKB_OK;  // every chunk is already in place
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != pg->device)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "peer group created on device %d, current %d",
                    pg->device, dev);
    int *err = device_error_word();
    if (!err) return fail(JKB_E_CUDA, fn, 0, 0, 0, "no device error word");
    for (int p = 0; p < pg->world; p++) {
        a.data[p] = pg->peer_base[p] + PEER_HDR;
        a.cnt[p] = reinterpret_cast<unsigned long long *>(pg->peer_base[p]);
    }
    a.expected = reinterpret_cast<unsigned long long *>(pg->base) + 1;
    a.arrivals = (unsigned long long)(pg->world - 1) * AG_CTAS;
    a.err = err;
    const cudaError_t le =
        launch_pdl(peer_allgather_kernel, dim3(AG_CTAS), dim3(AG_THREADS), 0, as_stream(stream), a);
    if (le != cudaSuccess) return fail_cuda(le, "peer_allgather_kernel");
    return check_launch("peer_allgather_kernel");
}

int jkb_peer_group_wait(jkb_peer_group *pg, uint64_t arrivals, void *stream) {
    if (!check_pg(pg)) return fail(JKB_E_INVALID, "peer_group_wait", 0, 0, 0, "null group");
    if (!pg->opened)
        return fail(JKB_E_INVALID, "peer_group_wait", 0, 0, 0, "peer group not opened");
    int *err = device_error_word();
    if (!err) return fail(JKB_E_CUDA, "peer_group_wait", 0, 0, 0, "no device error word");
    unsigned long long *cnt = reinterpret_cast<unsigned long long *>(pg->base);
    peer_wait_kernel<<<1, 32, 0, as_stream(stream)>>>(cnt, cnt + 1, (unsigned long long)arrivals,
                                                      err);
    return check_launch("peer_wait_kernel");
}

int jkb_peer_group_destroy(jkb_peer_group *pg) {
    if (!check_pg(pg)) return fail(JKB_E_INVALID, "peer_group_destroy", 0, 0, 0, "null group");
    pg->magic = 0;
    for (int p = 0; p < pg->world; p++)
        if (p != pg->rank && pg->peer_base[p]) cudaIpcCloseMemHandle(pg->peer_base[p]);
    cudaFree(pg->base);
    delete pg;
    return JKB_OK;
}

}  // extern "C"
