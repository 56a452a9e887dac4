// Peer groups: a one-kernel all-gather of output-row shards over NVLink.
//
// One process per GPU. Each rank's group owns one cudaMalloc allocation:
//   [0, 8)      arrival counter (u64): call signals received from peers, one per peer and call
//   [8, 16)     expected count (u64) of the arrival counter, advanced by each wait
//   [16, 24)    expected CTA signals per peer (u64), advanced by each all-gather or signal call
//   [64, 128)   CTA arrival counters (u64 per rank): entry p counts the CTA signals from rank p
//   [256, ...)  the output buffer handed to callers (`bytes` long), identical layout on every rank
// The ranks exchange CUDA IPC handles of these allocations and map each other's. The all-gather
// kernel copies this rank's chunks of the buffer to the same offsets in every peer's buffer with
// coalesced 16-byte stores over NVLink (plain stores; no multicast). Its CTA count follows the
// buffer size and the world size, so every rank launches the same grid. Each CTA then passes a
// CTA barrier, fences at system scope once and adds 1 to its own entry of every peer's CTA
// arrival counters (a release pattern: the fence, then relaxed adds); CTA 0 also adds 1 to
// every peer's arrival counter (the call's signal). CTA 0 then spins, with acquire loads and a
// 2 s bound, until every peer's entry has counted this call's CTAs and the call signals have
// arrived. Per-peer entries keep a fast peer's signals of the next call from standing in for a
// slow peer's signals of this one. The counts live on the device, so a captured CUDA graph
// stays correct across replays.
//
// Pushing groups: with push enabled, the GEMV kernels whose outputs lie in the group's buffer
// store every output element to the same offset in each peer's buffer as well (4-byte stores
// over NVLink, spread over the kernel's run) and fence them at system scope before they exit.
// The step then ends with jkb_peer_group_signal: the all-gather kernel with no chunks and one
// CTA, which only signals every peer and waits for their signals.
#include <atomic>
#include <cstring>
#include <mutex>

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
    bool push;  // registered in the pushing-group table
};

namespace jkb {

constexpr uint32_t PEER_MAGIC = 0x4A4B5031u;  // "JKP1"
constexpr size_t PEER_HDR = 256;              // counters and padding
constexpr unsigned long long PEER_WAIT_NS = 2000000000ull;
constexpr int AG_CTAS = 128;                  // most CTAs of an all-gather launch
constexpr int AG_THREADS = 256;
constexpr int AG_VEC = 4;                     // 16-byte loads in flight per thread

static bool check_pg(const jkb_peer_group *pg) { return pg && pg->magic == PEER_MAGIC; }

// The groups with push enabled, looked up by every GEMV launch while the count is non-zero.
constexpr int PUSH_MAX_GROUPS = 8;
std::mutex g_push_mu;
std::atomic<int> g_push_count{0};
jkb_peer_group *g_push[PUSH_MAX_GROUPS];

static void push_unregister(jkb_peer_group *pg) {
    std::lock_guard<std::mutex> lk(g_push_mu);
    for (int i = 0; i < PUSH_MAX_GROUPS; i++)
        if (g_push[i] == pg) {
            g_push[i] = nullptr;
            g_push_count.fetch_sub(1, std::memory_order_release);
        }
    pg->push = false;
}

int push_lookup(const void *lo, const void *hi, PushTarget *t, const char *who) {
    *t = PushTarget{};
    if (g_push_count.load(std::memory_order_acquire) == 0 || hi <= lo) return JKB_OK;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail_cuda(cudaGetLastError(), who);
    const uint8_t *l = static_cast<const uint8_t *>(lo), *h = static_cast<const uint8_t *>(hi);
    std::lock_guard<std::mutex> lk(g_push_mu);
    for (int i = 0; i < PUSH_MAX_GROUPS; i++) {
        const jkb_peer_group *pg = g_push[i];
        if (!pg || pg->device != dev) continue;
        const uint8_t *b = pg->base + PEER_HDR, *e = b + pg->bytes;
        if (h <= b || l >= e) continue;
        if (l < b || h > e)
            return fail(JKB_E_BOUNDS, who, (size_t)(l - b), (size_t)(h - l), pg->bytes,
                        "output range crosses the edge of a pushing peer group's %zu-byte buffer",
                        pg->bytes);
        for (int p = 0; p < pg->world; p++)
            if (p != pg->rank) t->delta[t->n++] = (long long)(pg->peer_base[p] - pg->base);
        t->group = pg;
        return JKB_OK;
    }
    return JKB_OK;
}

int push_reject(const void *lo, const void *hi, const char *who) {
    PushTarget t;
    int rc = push_lookup(lo, hi, &t, who);
    if (rc == JKB_OK && t.group)
        rc = fail(JKB_E_CAPABILITY, who, 0, 0, 0,
                  "output inside a pushing peer group's buffer: this entry point does not push "
                  "its outputs (use jkb_peer_group_allgather, or disable push)");
    return rc;
}

namespace {

// One all-gather launch. The chunks' 16-byte aligned bodies form one index space of 16-byte
// words (body_pre: prefix counts); their 4-byte heads and tails (up to 3 words each) are listed
// in w4. Both are laid out on the host.
struct AgArgs {
    int world, rank, nchunk, n4;
    unsigned long long body_off[JKB_PEER_MAX_CHUNKS];      // byte offset of chunk c's body
    unsigned long long body_pre[JKB_PEER_MAX_CHUNKS + 1];  // 16-byte words before chunk c's body
    unsigned long long w4[6 * JKB_PEER_MAX_CHUNKS];        // byte offsets of 4-byte words
    uint8_t *data[JKB_PEER_MAX_RANKS];                 // every rank's buffer (data region)
    unsigned long long *cnt[JKB_PEER_MAX_RANKS];       // every rank's arrival counter
    unsigned long long *ccnt[JKB_PEER_MAX_RANKS];      // every rank's CTA arrival counters
    unsigned long long *expected;                      // this rank's expected count
    unsigned long long *cexpected;                     // this rank's expected CTA signals
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

// Spins (thread 0 of the calling CTA) until every peer's entry of this rank's CTA arrival
// counters reaches *cexpected + add (which it stores back); bounded by PEER_WAIT_NS in total.
__device__ void bounded_cta_wait(const unsigned long long *entries, int world, int rank,
                                 unsigned long long *cexpected, unsigned long long add, int *err) {
    const unsigned long long target = *cexpected + add;
    *cexpected = target;
    unsigned long long t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (int p = 0; p < world; p++) {
        if (p == rank) continue;
        for (uint32_t i = 0;; i++) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(entries + p)
                         : "memory");
            if (v >= target) break;
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
    const unsigned long long nbody = a.body_pre[a.nchunk];
    // each thread loads up to AG_VEC words of the flat body index before storing any, so a
    // launch's L2 round trips overlap instead of following one another chunk by chunk
    for (size_t base = tid; base < nbody; base += AG_VEC * nthr) {
        uint4 v[AG_VEC];
        size_t o[AG_VEC];
#pragma unroll
        for (int u = 0; u < AG_VEC; u++) {
            const size_t i = base + (size_t)u * nthr;
            o[u] = ~(size_t)0;
            if (i < nbody) {
                int c = 0;
                while (c + 1 < a.nchunk && a.body_pre[c + 1] <= i) c++;
                o[u] = a.body_off[c] + ((i - a.body_pre[c]) << 4);
                v[u] = *reinterpret_cast<const uint4 *>(src + o[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < AG_VEC; u++)
            if (o[u] != ~(size_t)0)
                for (int p = 0; p < a.world; p++)
                    if (p != a.rank) *reinterpret_cast<uint4 *>(a.data[p] + o[u]) = v[u];
    }
    for (size_t i = tid; i < (size_t)a.n4; i += nthr) {
        const size_t o = a.w4[i];
        const uint32_t v = *reinterpret_cast<const uint32_t *>(src + o);
        for (int p = 0; p < a.world; p++)
            if (p != a.rank) *reinterpret_cast<uint32_t *>(a.data[p] + o) = v;
    }
    // The CTA barrier orders every thread's stores before thread 0's system-scope fence, which
    // is cumulative over them; the fence followed by each relaxed add is a release pattern for
    // the peer that reads the count. (A release add per peer would fence before each add, and
    // each fence waits for the previous add's NVLink round trip: with release adds from one CTA
    // the step's collection grew by about 2 us per added peer.)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < a.world; p++)
            if (p != a.rank)
                asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(a.ccnt[p] + a.rank)
                             : "memory");
        if (blockIdx.x == 0) {
            for (int p = 0; p < a.world; p++)
                if (p != a.rank)
                    asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(a.cnt[p])
                                 : "memory");
            bounded_cta_wait(a.ccnt[a.rank], a.world, a.rank, a.cexpected, gridDim.x, a.err);
            bounded_arrival_wait(a.cnt[a.rank], a.expected, a.arrivals, a.err);
        }
    }
}

__global__ void peer_wait_kernel(unsigned long long *cnt, unsigned long long *expected,
                                 unsigned long long arrivals, int *err) {
    if (threadIdx.x == 0) bounded_arrival_wait(cnt, expected, arrivals, err);
}

}  // namespace
}  // namespace jkb

using namespace jkb;

// CTAs of an all-gather launch: enough for one pass over a rank's share of the whole buffer
// (AG_VEC words a thread), 8 to AG_CTAS. It depends only on the buffer size and the world size,
// so every rank launches the same grid and expects as many CTA signals as it sends.
static int ag_ctas(const jkb_peer_group *pg) {
    const size_t words = pg->bytes / 16 / (size_t)pg->world;
    const size_t per_cta = (size_t)AG_THREADS * AG_VEC;
    size_t n = (words + per_cta - 1) / per_cta;
    if (n < 8) n = 8;
    if (n > (size_t)AG_CTAS) n = AG_CTAS;
    return (int)n;
}

// The all-gather kernel on `ctas` CTAs, each of which signals every peer once after its share
// of a's chunks (none for jkb_peer_group_signal).
static int launch_allgather(jkb_peer_group *pg, AgArgs &a, int ctas, void *stream,
                            const char *fn) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != pg->device)
        return fail(JKB_E_INVALID, fn, 0, 0, 0, "peer group created on device %d, current %d",
                    pg->device, dev);
    int *err = device_error_word();
    if (!err) return fail(JKB_E_CUDA, fn, 0, 0, 0, "no device error word");
    for (int p = 0; p < pg->world; p++) {
        a.data[p] = pg->peer_base[p] + PEER_HDR;
        a.cnt[p] = reinterpret_cast<unsigned long long *>(pg->peer_base[p]);
        a.ccnt[p] = reinterpret_cast<unsigned long long *>(pg->peer_base[p]) + 8;
    }
    a.expected = reinterpret_cast<unsigned long long *>(pg->base) + 1;
    a.cexpected = reinterpret_cast<unsigned long long *>(pg->base) + 2;
    a.arrivals = (unsigned long long)(pg->world - 1);  // one call signal from each peer
    a.err = err;
    const cudaError_t le =
        launch_pdl(peer_allgather_kernel, dim3(ctas), dim3(AG_THREADS), 0, as_stream(stream), a);
    if (le != cudaSuccess) return fail_cuda(le, "peer_allgather_kernel");
    return check_launch("peer_allgather_kernel");
}

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
        // 4-byte head up to a 16-byte boundary, 16-byte body, 4-byte tail
        const size_t off = offset[i], l = len[i];
        const size_t head = ((16 - (off & 15)) & 15) < l ? ((16 - (off & 15)) & 15) : l;
        const size_t body = (l - head) & ~(size_t)15;
        for (size_t o = off; o < off + head; o += 4) a.w4[a.n4++] = o;
        for (size_t o = off + head + body; o < off + l; o += 4) a.w4[a.n4++] = o;
        a.body_off[i] = off + head;
        a.body_pre[i + 1] = a.body_pre[i] + (body >> 4);
    }
    if (pg->world == 1) return JKB_OK;  // every chunk is already in place
    return launch_allgather(pg, a, ag_ctas(pg), stream, fn);
}

int jkb_peer_group_set_push(jkb_peer_group *pg, int enable) {
    static const char *fn = "peer_group_set_push";
    if (!check_pg(pg)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed group");
    if (!pg->opened) return fail(JKB_E_INVALID, fn, 0, 0, 0, "peer group not opened");
    if (!enable) {
        if (pg->push) push_unregister(pg);
        return JKB_OK;
    }
    std::lock_guard<std::mutex> lk(g_push_mu);
    if (pg->push) return JKB_OK;
    for (int i = 0; i < PUSH_MAX_GROUPS; i++)
        if (!g_push[i]) {
            g_push[i] = pg;
            pg->push = true;
            g_push_count.fetch_add(1, std::memory_order_release);
            return JKB_OK;
        }
    return fail(JKB_E_BOUNDS, fn, 0, PUSH_MAX_GROUPS, PUSH_MAX_GROUPS,
                "%d peer groups already push their outputs (limit)", PUSH_MAX_GROUPS);
}

int jkb_peer_group_signal(jkb_peer_group *pg, void *stream) {
    static const char *fn = "peer_group_signal";
    if (!check_pg(pg)) return fail(JKB_E_INVALID, fn, 0, 0, 0, "null or destroyed group");
    if (!pg->opened) return fail(JKB_E_INVALID, fn, 0, 0, 0, "peer group not opened");
    if (pg->world == 1) return JKB_OK;
    AgArgs a = {};
    a.world = pg->world;
    a.rank = pg->rank;
    a.nchunk = 0;
    return launch_allgather(pg, a, 1, stream, fn);
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
    if (pg->push) push_unregister(pg);
    pg->magic = 0;
    for (int p = 0; p < pg->world; p++)
        if (p != pg->rank && pg->peer_base[p]) cudaIpcCloseMemHandle(pg->peer_base[p]);
    cudaFree(pg->base);
    delete pg;
    return JKB_OK;
}

}  // extern "C"
