// Row-sharded GEMV over the GPUs of one node through peer memory (CUDA IPC over NVLink).
//
// The reference has no multi-GPU path.  The row-sharded configuration broadcasts x from rank 0 and
// gathers the y shards on every rank; instead of a broadcast and an all-gather launched around the
// GEMV, every rank maps the other ranks' shard buffers (cudaIpcOpenMemHandle) and the exchange is
// folded into the step:
//   1. rank 0 pushes x into every peer's x buffer (plain 16-byte stores over NVLink) and raises the
//      step's epoch in each peer's x flag (system-scope release);
//   2. every rank runs the GEMV of its rows; its CTAs first wait (bounded) for the x flag, and its
//      last CTA copies the finished y rows into every peer's gathered y and raises its done flag
//      there;
//   3. a one-warp kernel waits (bounded) until every peer's done flag carries the epoch.
// x and y are double-buffered by the parity of the step's epoch, so a step never overwrites data a
// peer may still be reading from the step before.  Every wait is bounded by %globaltimer; a
// timeout sets a status bit (l2d_shard_status) and the kernels return.  No TMA or bulk-copy load
// touches peer memory: only plain loads and stores.
#include "l2d_device.cuh"
#include "l2d_internal.h"

#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

namespace l2d {

struct GemvArgs;
int build_args(l2d_plan *p, const void *A, const void *x, void *y, int mode, GemvArgs *out, bool *split_out);
int launch_args(l2d_plan *p, const GemvArgs &a, bool split, void *stream);
int plan_device(const l2d_plan *p);
int64_t plan_rows(const l2d_plan *p);
const l2d_gemv_desc &plan_desc(const l2d_plan *p);
int shard_fill_args(GemvArgs *a, int world, int rank, unsigned long long epoch, const unsigned long long *x_flag,
                    uint8_t *const *peer_y, unsigned long long *const *peer_flags, int64_t y_off, int64_t y_bytes,
                    uint32_t *status, uint64_t timeout_ns);
size_t gemv_args_size();

namespace shard {

constexpr uint32_t kMagic = 0x4c32445du;  // "L2D]"
constexpr int kMaxWorld = 64;

struct Blob {
    uint32_t magic, version;
    int32_t pid, rank, world, device;
    int64_t bytes;
    uint64_t raw;  // device address in the exporting process (used when importer == exporter)
    cudaIpcMemHandle_t handle;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Rank 0: x into every peer's x buffer of this parity, then the epoch into each peer's x flag.
__global__ void k_push_x(const uint8_t *x, int64_t bytes, uint8_t *const *peer_x, unsigned long long *const *peer_flags,
                         int world, unsigned long long epoch) {
    const int64_t n16 = bytes / 16;
    for (int p = 1; p < world; ++p) {
        uint8_t *dst = peer_x[p];
        for (int64_t k = threadIdx.x; k < n16; k += blockDim.x)
            reinterpret_cast<uint4 *>(dst)[k] = reinterpret_cast<const uint4 *>(x)[k];
        for (int64_t k = n16 * 16 + threadIdx.x; k < bytes; k += blockDim.x) dst[k] = x[k];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x >= 1 && threadIdx.x < world) st_release_sys(peer_flags[threadIdx.x], epoch);
}

// Every rank: wait until each peer has pushed its y rows of this step (bounded).
__global__ void k_wait_done(const unsigned long long *flags, int world, int rank, unsigned long long epoch,
                            uint32_t *status, uint64_t timeout_ns) {
    if (threadIdx.x != 0) return;
    const uint64_t deadline = dev::globaltimer_ns() + timeout_ns;
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        while (ld_acquire_sys(flags + 1 + p) < epoch) {
            if (dev::globaltimer_ns() > deadline) {
                atomicOr(status, 2u);
                return;
            }
            __nanosleep(200);
        }
    }
}

// A rank without rows still publishes its (empty) part so the peers' waits end.
__global__ void k_raise_done(unsigned long long *const *peer_flags, int world, int rank, unsigned long long epoch) {
    if (threadIdx.x < world && threadIdx.x != rank) st_release_sys(peer_flags[threadIdx.x] + 1 + rank, epoch);
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace shard
}  // namespace l2d

struct l2d_shard {
    int device = 0, rank = 0, world = 1;
    int64_t M_total = 0, row0 = 0, rows = 0, N = 0;
    int dtype_in = 0, dtype_out = 0, eb_in = 4, eb_out = 4;
    uint64_t timeout_ns = 0;
    uint8_t *base = nullptr;  // local shared allocation
    size_t bytes = 0;
    size_t off_flags = 0, off_x[2] = {0, 0}, off_y[2] = {0, 0};
    std::vector<uint8_t *> peer;     // [world] peer bases in this process's address space
    std::vector<bool> opened;        // opened through IPC (closed on destroy)
    uint8_t *tables = nullptr;       // device: peer_x[2][world], peer_y[2][world], peer_flags[world], status
    bool connected = false;
    unsigned long long epoch = 0;
};

using namespace l2d;

namespace {

uint8_t **tab_x(l2d_shard *s, int par) { return reinterpret_cast<uint8_t **>(s->tables) + par * s->world; }
uint8_t **tab_y(l2d_shard *s, int par) { return reinterpret_cast<uint8_t **>(s->tables) + (2 + par) * s->world; }
unsigned long long **tab_flags(l2d_shard *s) {
    return reinterpret_cast<unsigned long long **>(s->tables) + 4 * s->world;
}
uint32_t *status_word(l2d_shard *s) { return reinterpret_cast<uint32_t *>(s->tables + 5 * s->world * sizeof(void *)); }

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int l2d_shard_create(int device, int rank, int world, int64_t M_total, int64_t row0, int64_t rows, int64_t N,
                     int dtype_in, int dtype_out, uint32_t timeout_ms, l2d_shard **out) {
    clear_error();
    if (!out) return set_error(L2D_ERR_INVALID, "shard_create: null output");
    *out = nullptr;
    if (world < 1 || world > shard::kMaxWorld || rank < 0 || rank >= world)
        return set_error(L2D_ERR_INVALID, "rank %d / world %d out of range", rank, world);
    if (M_total < 0 || row0 < 0 || rows < 0 || row0 + rows > M_total || N < 0 || !valid_dtype(dtype_in) ||
        !valid_dtype(dtype_out))
        return set_error(L2D_ERR_INVALID, "shard_create: bad rows, N or dtype");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", device);
    DeviceScope scope(device);
    l2d_shard *s = new (std::nothrow) l2d_shard();
    if (!s) return set_error(L2D_ERR_INVALID, "out of host memory");
    s->device = device;
    s->rank = rank;
    s->world = world;
    s->M_total = M_total;
    s->row0 = row0;
    s->rows = rows;
    s->N = N;
    s->dtype_in = dtype_in;
    s->dtype_out = dtype_out;
    s->eb_in = elem_bytes(dtype_in);
    s->eb_out = elem_bytes(dtype_out);
    s->timeout_ns = static_cast<uint64_t>(timeout_ms ? timeout_ms : 2000u) * 1000000ull;
    size_t off = 0;
    s->off_flags = off;
    off += shard::up256((1 + world) * sizeof(unsigned long long));
    for (int par = 0; par < 2; ++par) {
        s->off_x[par] = off;
        off += shard::up256(static_cast<size_t>(std::max<int64_t>(N, 1)) * s->eb_in);
    }
    for (int par = 0; par < 2; ++par) {
        s->off_y[par] = off;
        off += shard::up256(static_cast<size_t>(std::max<int64_t>(M_total, 1)) * s->eb_out);
    }
    s->bytes = off;
    cudaError_t e = cudaMalloc(&s->base, s->bytes);
    if (e == cudaSuccess) e = cudaMemset(s->base, 0, s->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&s->tables, 5 * world * sizeof(void *) + 256);
    if (e == cudaSuccess) e = cudaMemset(s->tables, 0, 5 * world * sizeof(void *) + 256);
    if (e != cudaSuccess) {
        if (s->base) cudaFree(s->base);
        delete s;
        return set_error(L2D_ERR_CUDA, "shard buffers: %s", cudaGetErrorString(e));
    }
    s->peer.assign(world, nullptr);
    s->opened.assign(world, false);
    s->peer[rank] = s->base;
    *out = s;
    return L2D_OK;
}

int l2d_shard_handle(const l2d_shard *s, void *blob, size_t cap, size_t *len) {
    clear_error();
    if (!s || !len) return set_error(L2D_ERR_INVALID, "shard_handle: null argument");
    *len = sizeof(shard::Blob);
    if (!blob) return L2D_OK;
    if (cap < sizeof(shard::Blob)) return set_error(L2D_ERR_INVALID, "handle buffer of %zu bytes < %zu", cap,
                                                    sizeof(shard::Blob));
    DeviceScope scope(s->device);
    shard::Blob b;
    std::memset(&b, 0, sizeof b);
    b.magic = shard::kMagic;
    b.version = 1;
    b.pid = static_cast<int32_t>(getpid());
    b.rank = s->rank;
    b.world = s->world;
    b.device = s->device;
    b.bytes = static_cast<int64_t>(s->bytes);
    b.raw = reinterpret_cast<uint64_t>(s->base);
    L2D_CUDA_TRY(cudaIpcGetMemHandle(&b.handle, s->base));
    std::memcpy(blob, &b, sizeof b);
    return L2D_OK;
}

int l2d_shard_connect(l2d_shard *s, const void *blobs, size_t blob_len) {
    clear_error();
    if (!s || !blobs || blob_len != sizeof(shard::Blob))
        return set_error(L2D_ERR_INVALID, "shard_connect: expected %d blobs of %zu bytes", s ? s->world : 0,
                         sizeof(shard::Blob));
    DeviceScope scope(s->device);
    const pid_t me = getpid();
    for (int r = 0; r < s->world; ++r) {
        shard::Blob b;
        std::memcpy(&b, static_cast<const uint8_t *>(blobs) + r * blob_len, sizeof b);
        if (b.magic != shard::kMagic || b.version != 1 || b.rank != r || b.world != s->world ||
            b.bytes != static_cast<int64_t>(s->bytes))
            return set_error(L2D_ERR_INVALID, "shard blob %d does not match this shard layout", r);
        if (r == s->rank) continue;
        if (s->peer[r]) continue;
        if (b.pid == static_cast<int32_t>(me)) {
            s->peer[r] = reinterpret_cast<uint8_t *>(b.raw);  // same process: the address is valid here
        } else {
            void *p = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&p, b.handle, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "opening rank %d's buffers: %s", r, cudaGetErrorString(e));
            s->peer[r] = static_cast<uint8_t *>(p);
            s->opened[r] = true;
        }
    }
    std::vector<uint8_t *> host(5 * s->world);
    for (int par = 0; par < 2; ++par)
        for (int r = 0; r < s->world; ++r) {
            host[par * s->world + r] = s->peer[r] + s->off_x[par];
            host[(2 + par) * s->world + r] = s->peer[r] + s->off_y[par];
        }
    for (int r = 0; r < s->world; ++r) host[4 * s->world + r] = s->peer[r] + s->off_flags;
    L2D_CUDA_TRY(cudaMemcpy(s->tables, host.data(), host.size() * sizeof(void *), cudaMemcpyHostToDevice));
    s->connected = true;
    return L2D_OK;
}

int l2d_shard_buffers(const l2d_shard *s, int parity, void **x, void **y) {
    if (!s || parity < 0 || parity > 1) return set_error(L2D_ERR_INVALID, "shard_buffers: bad argument");
    if (x) *x = s->base + s->off_x[parity];
    if (y) *y = s->base + s->off_y[parity];
    return L2D_OK;
}

int l2d_shard_next_parity(const l2d_shard *s) { return s ? static_cast<int>((s->epoch + 1) & 1ull) : -1; }

int l2d_gemv_sharded(l2d_plan *plan, l2d_shard *s, int mode, void *stream, int *parity) {
    clear_error();
    if (!plan || !s) return set_error(L2D_ERR_INVALID, "gemv_sharded: null plan or shard");
    if (!s->connected && s->world > 1) return set_error(L2D_ERR_INVALID, "gemv_sharded: shard not connected");
    const l2d_gemv_desc &d = plan_desc(plan);
    if (plan_device(plan) != s->device || plan_rows(plan) != s->rows || d.N != s->N || d.dtype_in != s->dtype_in ||
        d.dtype_out != s->dtype_out || d.batch > 1)
        return set_error(L2D_ERR_INVALID, "plan and shard disagree (device, rows, N, dtypes or batch)");
    DeviceScope scope(s->device);
    const unsigned long long e = ++s->epoch;
    const int par = static_cast<int>(e & 1ull);
    if (parity) *parity = par;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint8_t *x = s->base + s->off_x[par];
    uint8_t *yfull = s->base + s->off_y[par];
    if (s->world > 1 && s->rank == 0) {
        shard::k_push_x<<<1, 256, 0, cs>>>(x, s->N * s->eb_in, tab_x(s, par), tab_flags(s), s->world, e);
        L2D_CUDA_TRY(cudaGetLastError());
    }
    if (s->rows > 0) {
        std::vector<uint8_t> buf(gemv_args_size());
        GemvArgs *a = reinterpret_cast<GemvArgs *>(buf.data());
        bool split = false;
        int st = build_args(plan, d.A, x, yfull + s->row0 * s->eb_out, mode, a, &split);
        if (st != L2D_OK) return st;
        shard_fill_args(a, s->world, s->rank, e, reinterpret_cast<const unsigned long long *>(s->base + s->off_flags),
                        tab_y(s, par), tab_flags(s), s->row0 * s->eb_out, s->rows * s->eb_out, status_word(s),
                        s->timeout_ns);
        st = launch_args(plan, *a, split, stream);
        if (st != L2D_OK) return st;
    } else if (s->world > 1) {
        shard::k_raise_done<<<1, 64, 0, cs>>>(tab_flags(s), s->world, s->rank, e);
        L2D_CUDA_TRY(cudaGetLastError());
    }
    if (s->world > 1) {
        shard::k_wait_done<<<1, 32, 0, cs>>>(reinterpret_cast<const unsigned long long *>(s->base + s->off_flags),
                                             s->world, s->rank, e, status_word(s), s->timeout_ns);
        L2D_CUDA_TRY(cudaGetLastError());
    }
    return L2D_OK;
}

int l2d_shard_status(l2d_shard *s, uint32_t *status) {
    clear_error();
    if (!s || !status) return set_error(L2D_ERR_INVALID, "shard_status: null argument");
    DeviceScope scope(s->device);
    L2D_CUDA_TRY(cudaDeviceSynchronize());
    L2D_CUDA_TRY(cudaMemcpy(status, status_word(s), sizeof(uint32_t), cudaMemcpyDeviceToHost));
    return L2D_OK;
}

int l2d_shard_destroy(l2d_shard *s) {
    clear_error();
    if (!s) return L2D_OK;
    DeviceScope scope(s->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < s->world; ++r)
        if (s->opened[r]) cudaIpcCloseMemHandle(s->peer[r]);
    if (s->tables) cudaFree(s->tables);
    if (s->base) cudaFree(s->base);
    delete s;
    return L2D_OK;
}

}  // extern "C"
