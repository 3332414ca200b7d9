// Row-sharded GEMV over the GPUs of one node through peer memory (CUDA IPC over NVLink).
//
// The reference has no multi-GPU path.  The row-sharded configuration broadcasts x from rank 0 and
// gathers the y shards on every rank; instead of a broadcast and an all-gather launched around the
// GEMV, every rank maps the other ranks' exchange buffers (cudaIpcOpenMemHandle) and one GEMV
// launch per rank and step does the exchange while it computes.  Every transfer is a flagged
// 8-byte word -- 4 bytes of data and the step number -- written with one store into the reader's
// memory; the reader retries a word until its flag carries the step, so no fence, counter or
// barrier is on the way (the protocol NCCL calls LL):
//   * rank 0's CTAs store x into every peer's x words; the other ranks check them while they stage
//     x into shared memory;
//   * the CTA that finishes an interval of rows (the second of the two domain-group slots that
//     cover it) stores each final y into its own gathered y and into every peer's y words;
//   * at its end every CTA takes its share of the other ranks' rows from its own y words into the
//     gathered y.
// The words are double-buffered by the parity of the step number: a rank writes step e+2's words
// only after its step e+1, which needed the reader's step e+1 words, i.e. after the reader
// finished step e.  Every retry loop is bounded by %globaltimer; a timeout sets a status bit
// (l2d_shard_status) and the kernel returns.  No TMA or bulk-copy load touches peer memory: only
// plain stores and the readers' loads of their own memory.
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
int shard_fill_args(GemvArgs *a, const ShardArgs &sh);
size_t gemv_args_size();

namespace shard {

constexpr uint32_t kMagic = 0x4c32445du;  // "L2D]"
constexpr uint32_t kVersion = 3;
constexpr int kMaxWorld = 64;
constexpr int kIdleCtas = 32;   // grid of the step of a rank without rows

struct Blob {
    uint32_t magic, version;
    int32_t pid, rank, world, device;
    int64_t bytes, rows;
    int32_t reserved0, reserved1;
    uint64_t raw;  // device address in the exporting process (used when importer == exporter)
    cudaIpcMemHandle_t handle;
};

// The step of a rank without rows (M_total < world): rank 0 still pushes x as flagged words (as
// the GEMV prologue does), and every row of the gathered y comes from the peers' words.
__global__ void k_shard_idle(ShardArgs sh, const uint8_t *x, uint8_t *y_all, int eo) {
    const int lane = threadIdx.x;
    if (sh.rank == 0 && sh.world > 1) {
        const int64_t words = (sh.x_bytes + 3) / 4;
        const int64_t lo = words * blockIdx.x / gridDim.x, hi = words * (blockIdx.x + 1) / gridDim.x;
        const uint32_t flag = static_cast<uint32_t>(sh.epoch);
        for (int64_t w = lo + lane; w < hi; w += blockDim.x) {
            const uint32_t v = reinterpret_cast<const uint32_t *>(x)[w];
            for (int p = 1; p < sh.world; ++p)
                asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(sh.peer_xw[p] + w), "r"(v), "r"(flag)
                             : "memory");
        }
    }
    const uint32_t flag = static_cast<uint32_t>(sh.epoch);
    const uint64_t deadline = dev::globaltimer_ns() + sh.timeout_ns;
    const uint2 *yw = sh.peer_yw[sh.rank];
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + lane; g < sh.rows_all;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        uint32_t d, f;
        for (;;) {
            asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(d), "=r"(f) : "l"(yw + g) : "memory");
            if (f == flag) break;
            if (dev::globaltimer_ns() > deadline) {
                atomicOr(sh.status, 2u);
                return;
            }
            __nanosleep(64);
        }
        if (eo == 4) {
            reinterpret_cast<uint32_t *>(y_all)[g] = d;
        } else {
            reinterpret_cast<uint16_t *>(y_all)[g] = static_cast<uint16_t>(d);
        }
    }
}

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace shard
}  // namespace l2d

struct l2d_shard {
    int device = 0, rank = 0, world = 1;
    int64_t M_total = 0, row0 = 0, rows = 0, N = 0;
    int dtype_in = 0, dtype_out = 0, eb_in = 4, eb_out = 4;
    uint64_t timeout_ns = 0;
    uint8_t *base = nullptr;  // shared allocation: x[2], x words[2], y[2], y words[2]
    size_t bytes = 0;
    size_t off_x[2] = {0, 0}, off_xw[2] = {0, 0}, off_y[2] = {0, 0}, off_yw[2] = {0, 0};
    std::vector<uint8_t *> peer;  // [world] peer bases in this process's address space
    std::vector<bool> opened;     // opened through IPC (closed on destroy)
    // Local device tables: peer_xw[2][world], peer_yw[2][world] (pointers), status (u32).
    uint8_t *tables = nullptr;
    size_t off_status = 0, tables_bytes = 0;
    bool connected = false;
    unsigned long long epoch = 0;
};

using namespace l2d;

namespace {

uint2 **tab_xw(l2d_shard *s, int par) { return reinterpret_cast<uint2 **>(s->tables) + par * s->world; }
uint2 **tab_yw(l2d_shard *s, int par) { return reinterpret_cast<uint2 **>(s->tables) + (2 + par) * s->world; }
uint32_t *status_word(l2d_shard *s) { return reinterpret_cast<uint32_t *>(s->tables + s->off_status); }

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

ShardArgs shard_args(l2d_shard *s, int par, unsigned long long e) {
    ShardArgs sh;
    std::memset(&sh, 0, sizeof sh);
    sh.world = s->world;
    sh.rank = s->rank;
    sh.epoch = e;
    sh.peer_xw = tab_xw(s, par);
    sh.peer_yw = tab_yw(s, par);
    sh.row0 = s->row0;
    sh.rows_all = s->M_total;
    sh.x_bytes = s->N * s->eb_in;
    sh.status = status_word(s);
    sh.timeout_ns = s->timeout_ns;
    return sh;
}

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
    for (int par = 0; par < 2; ++par) {
        s->off_x[par] = off;
        off += shard::up256(static_cast<size_t>(std::max<int64_t>(N, 1)) * s->eb_in);
    }
    const size_t words = (static_cast<size_t>(std::max<int64_t>(N, 1)) * s->eb_in + 3) / 4;
    for (int par = 0; par < 2; ++par) {
        s->off_xw[par] = off;
        off += shard::up256(words * sizeof(uint2));
    }
    for (int par = 0; par < 2; ++par) {
        s->off_y[par] = off;
        off += shard::up256(static_cast<size_t>(std::max<int64_t>(M_total, 1)) * s->eb_out);
    }
    for (int par = 0; par < 2; ++par) {
        s->off_yw[par] = off;
        off += shard::up256(static_cast<size_t>(std::max<int64_t>(M_total, 1)) * sizeof(uint2));
    }
    s->bytes = off;
    s->off_status = 4 * world * sizeof(void *);
    s->tables_bytes = s->off_status + 16;
    cudaError_t e = cudaMalloc(&s->base, s->bytes);
    if (e == cudaSuccess) e = cudaMemset(s->base, 0, s->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&s->tables, s->tables_bytes);
    if (e == cudaSuccess) e = cudaMemset(s->tables, 0, s->tables_bytes);
    if (e != cudaSuccess) {
        if (s->tables) cudaFree(s->tables);
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
    if (cap < sizeof(shard::Blob))
        return set_error(L2D_ERR_INVALID, "handle buffer of %zu bytes < %zu", cap, sizeof(shard::Blob));
    DeviceScope scope(s->device);
    shard::Blob b;
    std::memset(&b, 0, sizeof b);
    b.magic = shard::kMagic;
    b.version = shard::kVersion;
    b.pid = static_cast<int32_t>(getpid());
    b.rank = s->rank;
    b.world = s->world;
    b.device = s->device;
    b.bytes = static_cast<int64_t>(s->bytes);
    b.rows = s->rows;
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

    int64_t rows_sum = 0;
    for (int r = 0; r < s->world; ++r) {
        shard::Blob b;
        std::memcpy(&b, static_cast<const uint8_t *>(blobs) + r * blob_len, sizeof b);
        if (b.magic != shard::kMagic || b.version != shard::kVersion || b.rank != r || b.world != s->world ||
            b.bytes != static_cast<int64_t>(s->bytes) || b.rows < 0)
            return set_error(L2D_ERR_INVALID, "shard blob %d does not match this shard layout", r);
        rows_sum += b.rows;
        if (r == s->rank || s->peer[r]) continue;
        if (b.pid == static_cast<int32_t>(me)) {
            s->peer[r] = reinterpret_cast<uint8_t *>(b.raw);  // same process: the address is valid here
        } else {
            void *p = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&p, b.handle, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess)
                return set_error(L2D_ERR_CUDA, "opening rank %d's buffers: %s", r, cudaGetErrorString(e));
            s->peer[r] = static_cast<uint8_t *>(p);
            s->opened[r] = true;
        }
    }
    if (rows_sum != s->M_total)
        return set_error(L2D_ERR_INVALID, "the ranks' rows add up to %lld, not M_total = %lld",
                         static_cast<long long>(rows_sum), static_cast<long long>(s->M_total));
    std::vector<uint8_t *> host(4 * s->world);
    for (int par = 0; par < 2; ++par)
        for (int r = 0; r < s->world; ++r) {
            host[par * s->world + r] = s->peer[r] + s->off_xw[par];
            host[(2 + par) * s->world + r] = s->peer[r] + s->off_yw[par];
        }
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
    if (!s) return set_error(L2D_ERR_INVALID, "gemv_sharded: null shard");
    if (!s->connected) return set_error(L2D_ERR_INVALID, "gemv_sharded: shard not connected");
    if (s->rows > 0) {
        if (!plan) return set_error(L2D_ERR_INVALID, "gemv_sharded: null plan");
        const l2d_gemv_desc &d = plan_desc(plan);
        if (plan_device(plan) != s->device || plan_rows(plan) != s->rows || d.N != s->N ||
            d.dtype_in != s->dtype_in || d.dtype_out != s->dtype_out || d.batch > 1)
            return set_error(L2D_ERR_INVALID, "plan and shard disagree (device, rows, N, dtypes or batch)");
    }
    DeviceScope scope(s->device);
    const unsigned long long e = s->epoch + 1;
    const int par = static_cast<int>(e & 1ull);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const ShardArgs sh = shard_args(s, par, e);
    if (s->rows > 0) {
        std::vector<uint8_t> buf(gemv_args_size());
        GemvArgs *a = reinterpret_cast<GemvArgs *>(buf.data());
        bool split = false;
        const l2d_gemv_desc &d = plan_desc(plan);
        int st = build_args(plan, d.A, s->base + s->off_x[par], s->base + s->off_y[par] + s->row0 * s->eb_out, mode,
                            a, &split);
        if (st == L2D_OK) st = shard_fill_args(a, sh);
        if (st == L2D_OK) st = launch_args(plan, *a, split, stream);
        if (st != L2D_OK) return st;
    } else if (s->world > 1) {
        shard::k_shard_idle<<<shard::kIdleCtas, 256, 0, cs>>>(sh, s->base + s->off_x[par], s->base + s->off_y[par],
                                                            s->eb_out);
        L2D_CUDA_TRY(cudaGetLastError());
    }
    s->epoch = e;  // only a launched step advances the step number (all ranks must stay in step)
    if (parity) *parity = par;
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
