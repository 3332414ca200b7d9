// L2-domain-aware GEMV for sm_100a (y = A.x, fp32 accumulation).
//
// Reference: applications/gemv/src/gemv_k1024_persistent_subwarp.cu:141-231.  The reference runs a
// persistent grid of one 512-thread CTA per SM; an SM of side s walks a host-built list of whole
// rows homed on side s, one warp per row (K = 1024 fp32 = one 4 KiB granule, so a row never
// crosses domains), float4 loads, shuffle reduction.
//
// This kernel keeps the persistent-grid / one-CTA-per-SM shape but is rebuilt for Blackwell:
//  * Work is split at 512-byte windows (absolute address alignment), not rows: rows of the
//    BASELINE shapes are 8-32 KiB and cross many domain granules.  A window lies inside one
//    granule whenever the granule is >= 512 B, and its domain is computed in the kernel from the
//    probed XOR mask and the per-2-MiB-page attr bits (the reference's predictor), so no row lists
//    are read.  The SMs of domain d stream exactly the windows homed in d (AWARE), the other
//    domain's (SWAPPED), or a pseudo-random half at the same granule size (OBLIVIOUS).
//  * Per row, each domain group produces one fp32 partial; the second group to arrive (per-row
//    counter) adds them as part[0] + part[1] and stores y.  The sum is therefore deterministic.
//  * Each lane issues U independent 16-byte streaming loads (ld.global.nc.L1::no_allocate) per
//    step, gathered across windows with a 64-window ballot mask, so the loads in flight do not
//    drain at granule boundaries.  x is read through L1 (ld.global.nc), where it stays resident.
//  * Rows are blocked per slot (one slot per SM) and interleaved over the CTA's warps.  Slots are
//    claimed with a per-call epoch: a CTA whose SM slot is already taken (two CTAs on one SM) takes
//    any unclaimed slot, and the last CTA to finish processes slots nobody claimed, so every row
//    is computed exactly once whatever the block scheduler does.  No wait anywhere.
#include "l2d_device.cuh"
#include "l2d_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <vector>

namespace l2d {

constexpr int kWindowShift = 9;  // 512-byte windows: one 16-byte piece per lane
constexpr int kThreads = 512;
constexpr int kUnroll = 8;

struct GemvArgs {
    const uint8_t *A;
    const uint8_t *x;
    uint8_t *y;
    int64_t M;
    int64_t row_bytes;
    int64_t lda_bytes;
    int64_t stride_a_bytes;
    int64_t stride_x_bytes;
    int64_t stride_y_elems;
    int64_t rows_total;
    const uint8_t *region_base;   // 512-B aligned (2 MiB aligned when the attr table is used)
    const uint32_t *attr_bits;    // per 2 MiB page of the region, 32 pages per word
    uint32_t mask;
    int gran_shift;
    int dom_kind;                 // 0 = probed XOR model, 1 = hash of the granule index
    int flip;                     // 1 = swapped control
    const int32_t *sm_slot;       // [kMaxSmid] slot of each SM, -1 = none
    int n_slots;
    int n_dom0;
    int n_dom1;
    float *part;                  // [2 * rows_total]
    uint32_t *cnt;                // [rows_total], zero between calls
    unsigned long long *claim;    // [n_slots] epoch of the last claim
    unsigned long long *ctl;      // [0] epoch, [1] CTAs done, [2] fallback claims
};

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ld_cached16(const void *p) {
    uint4 v;
    asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t mix_granule(uint64_t g) {
    uint32_t h = static_cast<uint32_t>(g) ^ static_cast<uint32_t>(g >> 32) * 0x9e3779b9u;
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}

// Domain of the 512-byte window w (region-relative index) as seen by the split.
__device__ __forceinline__ int window_dom(const GemvArgs &a, uint64_t w) {
    uint64_t wa = w << kWindowShift;
    int d;
    if (a.dom_kind == 0) {
        uint64_t page = wa >> kPageShift;
        int attr = (__ldg(a.attr_bits + (page >> 5)) >> (page & 31)) & 1;
        d = (__popc(static_cast<uint32_t>(wa) & a.mask) & 1) ^ attr;
    } else {
        d = mix_granule(wa >> a.gran_shift) & 1;
    }
    return d ^ a.flip;
}

template <int DT> struct Dot;

template <> struct Dot<L2D_F32> {
    static __device__ __forceinline__ float run(const uint4 &a, const uint4 &x, float acc) {
        acc = fmaf(__uint_as_float(a.x), __uint_as_float(x.x), acc);
        acc = fmaf(__uint_as_float(a.y), __uint_as_float(x.y), acc);
        acc = fmaf(__uint_as_float(a.z), __uint_as_float(x.z), acc);
        acc = fmaf(__uint_as_float(a.w), __uint_as_float(x.w), acc);
        return acc;
    }
    static __device__ __forceinline__ float elem(const uint8_t *p) { return *reinterpret_cast<const float *>(p); }
};

__device__ __forceinline__ float2 h2f(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2 *>(&u);
    return __half22float2(h);
}

template <> struct Dot<L2D_F16> {
    static __device__ __forceinline__ float run(const uint4 &a, const uint4 &x, float acc) {
        float2 a0 = h2f(a.x), a1 = h2f(a.y), a2 = h2f(a.z), a3 = h2f(a.w);
        float2 x0 = h2f(x.x), x1 = h2f(x.y), x2 = h2f(x.z), x3 = h2f(x.w);
        acc = fmaf(a0.x, x0.x, acc);
        acc = fmaf(a0.y, x0.y, acc);
        acc = fmaf(a1.x, x1.x, acc);
        acc = fmaf(a1.y, x1.y, acc);
        acc = fmaf(a2.x, x2.x, acc);
        acc = fmaf(a2.y, x2.y, acc);
        acc = fmaf(a3.x, x3.x, acc);
        acc = fmaf(a3.y, x3.y, acc);
        return acc;
    }
    static __device__ __forceinline__ float elem(const uint8_t *p) {
        return __half2float(*reinterpret_cast<const __half *>(p));
    }
};

// bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

template <> struct Dot<L2D_BF16> {
    static __device__ __forceinline__ float run(const uint4 &a, const uint4 &x, float acc) {
        acc = fmaf(bf_lo(a.x), bf_lo(x.x), acc);
        acc = fmaf(bf_hi(a.x), bf_hi(x.x), acc);
        acc = fmaf(bf_lo(a.y), bf_lo(x.y), acc);
        acc = fmaf(bf_hi(a.y), bf_hi(x.y), acc);
        acc = fmaf(bf_lo(a.z), bf_lo(x.z), acc);
        acc = fmaf(bf_hi(a.z), bf_hi(x.z), acc);
        acc = fmaf(bf_lo(a.w), bf_lo(x.w), acc);
        acc = fmaf(bf_hi(a.w), bf_hi(x.w), acc);
        return acc;
    }
    static __device__ __forceinline__ float elem(const uint8_t *p) {
        return __uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t *>(p)) << 16);
    }
};

template <int DT> __device__ __forceinline__ void store_out(uint8_t *y, float v);
template <> __device__ __forceinline__ void store_out<L2D_F32>(uint8_t *y, float v) { *reinterpret_cast<float *>(y) = v; }
template <> __device__ __forceinline__ void store_out<L2D_F16>(uint8_t *y, float v) {
    *reinterpret_cast<__half *>(y) = __float2half_rn(v);
}
template <> __device__ __forceinline__ void store_out<L2D_BF16>(uint8_t *y, float v) {
    *reinterpret_cast<__nv_bfloat16 *>(y) = __float2bfloat16_rn(v);
}

// Partial piece at the end of a row (N * elem_bytes not a multiple of 16): element by element.
template <int DT_IN>
__device__ __forceinline__ float tail_piece(const uint8_t *ap, const uint8_t *xp, int nbytes, float acc) {
    constexpr int eb = DT_IN == L2D_F32 ? 4 : 2;
    for (int o = 0; o < nbytes; o += eb) acc = fmaf(Dot<DT_IN>::elem(ap + o), Dot<DT_IN>::elem(xp + o), acc);
    return acc;
}

template <int DT_IN, int DT_OUT, bool SPLIT>
__device__ __forceinline__ void gemv_row(const GemvArgs &a, int64_t row, int grp, int lane) {
    constexpr int eo = DT_OUT == L2D_F32 ? 4 : 2;
    const int64_t b = row / a.M;
    const int64_t i = row - b * a.M;
    const uint8_t *rowp = a.A + b * a.stride_a_bytes + i * a.lda_bytes;
    const uint8_t *xrow = a.x + b * a.stride_x_bytes;
    uint8_t *yp = a.y + (b * a.stride_y_elems + i) * eo;
    const uint64_t rs = static_cast<uint64_t>(rowp - a.region_base);
    const uint64_t re = rs + static_cast<uint64_t>(a.row_bytes);
    const uint64_t w0 = rs >> kWindowShift;
    const uint64_t w1 = (re + (1u << kWindowShift) - 1) >> kWindowShift;
    if (w0 == w1) {  // N == 0: y = 0, written once
        if (lane == 0 && grp == 0) store_out<DT_OUT>(yp, 0.0f);
        return;
    }
    float acc0 = 0.0f, acc1 = 0.0f;
    bool saw_mine = false, saw_other = false;
    for (uint64_t wb = w0; wb < w1; wb += 64) {
        uint64_t bits;
        if (!SPLIT) {
            uint64_t n = w1 - wb;
            bits = n >= 64 ? ~0ull : ((1ull << n) - 1);
        } else {
            const uint64_t wa = wb + lane, wb2 = wb + 32 + lane;
            const bool ina = wa < w1, inb = wb2 < w1;
            const bool ma = ina && window_dom(a, wa) == grp;
            const bool mb = inb && window_dom(a, wb2) == grp;
            const uint32_t ba = __ballot_sync(0xffffffffu, ma), bb = __ballot_sync(0xffffffffu, mb);
            const uint32_t oa = __ballot_sync(0xffffffffu, ina && !ma), ob = __ballot_sync(0xffffffffu, inb && !mb);
            bits = static_cast<uint64_t>(ba) | (static_cast<uint64_t>(bb) << 32);
            saw_other |= (oa | ob) != 0u;
        }
        saw_mine |= bits != 0ull;
        while (bits) {
            int widx[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                widx[u] = bits ? __ffsll(static_cast<long long>(bits)) - 1 : -1;
                bits &= bits - 1;
            }
            uint4 av[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                av[u] = make_uint4(0u, 0u, 0u, 0u);
                if (widx[u] >= 0) {
                    const uint64_t pa = ((wb + widx[u]) << kWindowShift) + static_cast<uint64_t>(lane) * 16u;
                    if (pa >= rs && pa + 16 <= re) av[u] = ld_stream16(a.region_base + pa);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                if (widx[u] >= 0) {
                    const uint64_t pa = ((wb + widx[u]) << kWindowShift) + static_cast<uint64_t>(lane) * 16u;
                    if (pa >= rs && pa + 16 <= re) {
                        const uint4 xv = ld_cached16(xrow + (pa - rs));
                        if (u & 1) acc1 = Dot<DT_IN>::run(av[u], xv, acc1);
                        else acc0 = Dot<DT_IN>::run(av[u], xv, acc0);
                    } else if (pa >= rs && pa < re) {
                        acc0 = tail_piece<DT_IN>(a.region_base + pa, xrow + (pa - rs), static_cast<int>(re - pa), acc0);
                    }
                }
            }
        }
    }
    float acc = acc0 + acc1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane != 0 || !saw_mine) return;
    if (!SPLIT || !saw_other) {
        store_out<DT_OUT>(yp, acc);
        return;
    }
    // Both domain groups own part of this row: publish the partial, the second arriver combines.
    volatile float *part = a.part;
    part[static_cast<int64_t>(grp) * a.rows_total + row] = acc;
    __threadfence();
    const uint32_t old = atomicAdd(a.cnt + row, 1u);
    if (old == 1u) {
        __threadfence();
        const float other = part[static_cast<int64_t>(grp ^ 1) * a.rows_total + row];
        store_out<DT_OUT>(yp, acc + other);  // commutative: identical bits whichever arrives last
        a.cnt[row] = 0u;
    }
}

template <int DT_IN, int DT_OUT, bool SPLIT>
__device__ __forceinline__ void run_slot(const GemvArgs &a, int slot, int warp, int nwarps, int lane) {
    int grp = 0, idx = slot, n_group = a.n_slots;
    if (SPLIT) {
        grp = slot >= a.n_dom0;
        idx = grp ? slot - a.n_dom0 : slot;
        n_group = grp ? a.n_dom1 : a.n_dom0;
    }
    const int64_t r0 = a.rows_total * idx / n_group;
    const int64_t r1 = a.rows_total * (idx + 1) / n_group;
    for (int64_t row = r0 + warp; row < r1; row += nwarps) gemv_row<DT_IN, DT_OUT, SPLIT>(a, row, grp, lane);
}

// Claims the first slot whose claim epoch is older than E (any domain); -1 if none is left.
__device__ __forceinline__ int claim_any(const GemvArgs &a, unsigned long long E) {
    for (int t = 0; t < a.n_slots; ++t)
        if (atomicMax(a.claim + t, E) < E) return t;
    return -1;
}

template <int DT_IN, int DT_OUT, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(GemvArgs a) {
    __shared__ int s_slot;
    __shared__ int s_last;
    __shared__ unsigned long long s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    if (tid == 0) {
        const unsigned long long E = *reinterpret_cast<volatile unsigned long long *>(a.ctl) + 1ull;
        s_epoch = E;
        const uint32_t sm = dev::smid();
        const int home = sm < static_cast<uint32_t>(kMaxSmid) ? a.sm_slot[sm] : -1;
        int got = -1;
        if (home >= 0 && atomicMax(a.claim + home, E) < E) {
            got = home;
        } else {
            got = claim_any(a, E);
            if (got >= 0) atomicAdd(a.ctl + 2, 1ull);
        }
        s_slot = got;
    }
    __syncthreads();
    if (s_slot >= 0) run_slot<DT_IN, DT_OUT, SPLIT>(a, s_slot, warp, nwarps, lane);
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned long long done = atomicAdd(a.ctl + 1, 1ull);
        s_last = done == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    // Last CTA: slots whose SM never hosted a CTA of this launch.
    for (;;) {
        if (tid == 0) {
            const int got = claim_any(a, s_epoch);
            if (got >= 0) atomicAdd(a.ctl + 2, 1ull);
            s_slot = got;
        }
        __syncthreads();
        const int t = s_slot;
        if (t < 0) break;
        run_slot<DT_IN, DT_OUT, SPLIT>(a, t, warp, nwarps, lane);
        __syncthreads();
    }
    if (tid == 0) {
        a.ctl[1] = 0ull;
        __threadfence();
        *reinterpret_cast<volatile unsigned long long *>(a.ctl) = s_epoch;
    }
}

using KernelFn = void (*)(GemvArgs);

template <int DI, int DO> KernelFn pick_split(bool split) {
    return split ? k_gemv<DI, DO, true> : k_gemv<DI, DO, false>;
}

template <int DI> KernelFn pick_out(int dout, bool split) {
    switch (dout) {
    case L2D_F32: return pick_split<DI, L2D_F32>(split);
    case L2D_F16: return pick_split<DI, L2D_F16>(split);
    default: return pick_split<DI, L2D_BF16>(split);
    }
}

KernelFn pick_kernel(int din, int dout, bool split) {
    switch (din) {
    case L2D_F32: return pick_out<L2D_F32>(dout, split);
    case L2D_F16: return pick_out<L2D_F16>(dout, split);
    default: return pick_out<L2D_BF16>(dout, split);
    }
}

// ---------------------------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------------------------

int probe_sm_domains_impl(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts,
                          l2d_sm_probe_report *report, uint32_t *raw, size_t raw_cap, size_t *raw_len);
int probe_addr_domains_impl(int device, const uint8_t *base, size_t valid_bytes, const int *sm_map, int num_sm,
                            uint32_t *mask, int *attr, size_t cap_pages, size_t *num_pages_out,
                            const l2d_probe_opts *opts, l2d_addr_probe_report *report, uint32_t *raw,
                            size_t raw_cap, size_t *raw_len);

namespace {

std::mutex g_sm_cache_mu;
std::map<int, std::vector<int>> g_sm_cache;  // device -> SM domain map

int cached_sm_map(int device, std::vector<int> &out) {
    {
        std::lock_guard<std::mutex> lk(g_sm_cache_mu);
        auto it = g_sm_cache.find(device);
        if (it != g_sm_cache.end()) {
            out = it->second;
            return L2D_OK;
        }
    }
    int n = 0;
    int st = probe_sm_domains_impl(device, nullptr, 0, &n, nullptr, nullptr, nullptr, 0, nullptr);
    if (st != L2D_OK) return st;
    std::vector<int> map(n, 0);
    st = probe_sm_domains_impl(device, map.data(), n, &n, nullptr, nullptr, nullptr, 0, nullptr);
    if (st != L2D_OK) return st;
    std::lock_guard<std::mutex> lk(g_sm_cache_mu);
    g_sm_cache[device] = map;
    out = map;
    return L2D_OK;
}

// Allocation containing p, through the driver entry point (no link-time libcuda dependency).
typedef int (*PFN_memGetAddressRange)(unsigned long long *, size_t *, unsigned long long);
int alloc_range(const void *p, uint64_t *base, uint64_t *size) {
    static PFN_memGetAddressRange fn = nullptr;
    if (!fn) {
        void *sym = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !sym)
            return set_error(L2D_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
        fn = reinterpret_cast<PFN_memGetAddressRange>(sym);
    }
    unsigned long long b = 0;
    size_t s = 0;
    int r = fn(&b, &s, reinterpret_cast<unsigned long long>(p));
    if (r != 0) return set_error(L2D_ERR_INVALID, "A is not a device allocation (cuMemGetAddressRange error %d)", r);
    *base = b;
    *size = s;
    return L2D_OK;
}

}  // namespace

}  // namespace l2d

struct l2d_plan {
    l2d_gemv_desc desc{};
    int device = 0;
    int64_t rows_total = 0;
    int eb_in = 4, eb_out = 4;
    bool has_domains = false;
    int num_sm = 0;
    std::vector<int> sm_domain;
    uint32_t mask = 0;
    std::vector<int> attr;
    const uint8_t *region_base = nullptr;  // 2 MiB aligned base of the attr table
    const uint8_t *stream_base = nullptr;  // 512 B aligned base for the unsplit kernel
    int gran_shift = l2d::kPageShift;
    int n_dom[2] = {0, 0};
    int n_slots = 0;
    int64_t domain_bytes[2] = {0, 0};
    int64_t split_rows = 0;
    void *dev_block = nullptr;
    size_t dev_bytes = 0;
    int32_t *d_sm_slot = nullptr;
    uint32_t *d_attr_bits = nullptr;
    float *d_part = nullptr;
    uint32_t *d_cnt = nullptr;
    unsigned long long *d_claim = nullptr;
    unsigned long long *d_ctl = nullptr;
};

using namespace l2d;

namespace {

int64_t row_offset_bytes(const l2d_plan &p, int64_t row) {
    const int64_t b = row / p.desc.M, i = row - b * p.desc.M;
    return (b * p.desc.stride_a + i * p.desc.lda) * p.eb_in;
}

// Bytes of A homed in each domain and the number of rows touching both (for the stats report).
void domain_census(l2d_plan &p) {
    p.domain_bytes[0] = p.domain_bytes[1] = 0;
    p.split_rows = 0;
    if (!p.has_domains || p.rows_total == 0) return;
    const uint64_t A = reinterpret_cast<uint64_t>(p.desc.A), base = reinterpret_cast<uint64_t>(p.region_base);
    const int64_t rb = p.desc.N * p.eb_in;
    const int64_t sample_rows = std::min<int64_t>(p.rows_total, 65536);
    const int64_t step = std::max<int64_t>(1, p.rows_total / sample_rows);
    int64_t sampled = 0;
    for (int64_t r = 0; r < p.rows_total; r += step, ++sampled) {
        uint64_t s = A + row_offset_bytes(p, r) - base, e = s + rb;
        bool seen[2] = {false, false};
        for (uint64_t w = s >> 9; w < (e + 511) >> 9; ++w) {
            uint64_t wa = w << 9;
            int d = l2d::parity_domain(p.mask, wa, p.attr[wa >> kPageShift]);
            uint64_t lo = std::max(wa, s), hi = std::min(wa + 512, e);
            p.domain_bytes[d] += static_cast<int64_t>(hi - lo);
            seen[d] = true;
        }
        p.split_rows += seen[0] && seen[1];
    }
    if (sampled && step > 1) {
        double scale = static_cast<double>(p.rows_total) / sampled;
        p.domain_bytes[0] = static_cast<int64_t>(p.domain_bytes[0] * scale);
        p.domain_bytes[1] = static_cast<int64_t>(p.domain_bytes[1] * scale);
        p.split_rows = static_cast<int64_t>(p.split_rows * scale);
    }
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

extern "C" {

int l2d_plan_create(const l2d_gemv_desc *desc_in, const l2d_domain_map *map, l2d_plan **out) {
    clear_error();
    if (!desc_in || !out) return set_error(L2D_ERR_INVALID, "plan_create: null argument");
    *out = nullptr;
    l2d_gemv_desc d = *desc_in;
    if (d.M < 0 || d.N < 0) return set_error(L2D_ERR_INVALID, "M and N must be >= 0");
    if (!valid_dtype(d.dtype_in) || !valid_dtype(d.dtype_out)) return set_error(L2D_ERR_INVALID, "bad dtype");
    if (d.lda == 0) d.lda = d.N;
    if (d.lda < d.N) return set_error(L2D_ERR_INVALID, "lda %lld < N %lld", (long long)d.lda, (long long)d.N);
    if (d.batch <= 0) d.batch = 1;
    if (d.stride_a == 0) d.stride_a = d.M * d.lda;
    if (d.stride_x == 0) d.stride_x = d.N;
    if (d.stride_y == 0) d.stride_y = d.M;
    if (d.batch > 1 && (d.stride_a < d.M * d.lda || d.stride_x < d.N || d.stride_y < d.M))
        return set_error(L2D_ERR_INVALID, "batch strides overlap");
    if (d.M > 0 && d.batch > (int64_t(1) << 40) / std::max<int64_t>(d.M, 1))
        return set_error(L2D_ERR_INVALID, "batch * M too large");
    const int eb = elem_bytes(d.dtype_in);
    if (((d.lda * eb) & 15) || ((d.stride_a * eb) & 15) || ((d.stride_x * eb) & 15))
        return set_error(L2D_ERR_UNSUPPORTED, "lda, stride_a and stride_x must be multiples of 16 bytes");
    if (reinterpret_cast<uintptr_t>(d.A) & 15) return set_error(L2D_ERR_UNSUPPORTED, "A must be 16-byte aligned");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (d.device < 0 || d.device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", d.device);
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d.device);
    struct Restore {
        int prev;
        ~Restore() {
            if (prev >= 0) cudaSetDevice(prev);
        }
    } restore{prev};

    l2d_plan *p = new (std::nothrow) l2d_plan();
    if (!p) return set_error(L2D_ERR_INVALID, "out of host memory");
    p->desc = d;
    p->device = d.device;
    p->rows_total = d.batch * d.M;
    p->eb_in = eb;
    p->eb_out = elem_bytes(d.dtype_out);
    int st = L2D_OK;
    const uint64_t A = reinterpret_cast<uint64_t>(d.A);
    const uint64_t span = p->rows_total ? static_cast<uint64_t>(row_offset_bytes(*p, p->rows_total - 1) + d.N * eb) : 0;
    p->stream_base = reinterpret_cast<const uint8_t *>(A & ~uint64_t(511));
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&p->num_sm, cudaDevAttrMultiProcessorCount, d.device));

    // Domain model: the caller's, or probed now (SM map cached per device, address model of A).
    if (map) {
        if (!map->sm_domain || map->num_sm != p->num_sm) {
            delete p;
            return set_error(L2D_ERR_INVALID, "domain map has %d SMs, device has %d", map->num_sm, p->num_sm);
        }
        p->sm_domain.assign(map->sm_domain, map->sm_domain + map->num_sm);
        p->mask = map->mask;
        const uint64_t base = reinterpret_cast<uint64_t>(map->base);
        if (base % kPageBytes || !map->attr || base > A || A + span > base + map->num_pages * kPageBytes) {
            delete p;
            return set_error(L2D_ERR_INVALID, "domain map region does not cover A");
        }
        p->region_base = reinterpret_cast<const uint8_t *>(base);
        p->attr.assign(map->attr, map->attr + map->num_pages);
        p->has_domains = true;
    } else if (span > 0 && !(d.flags & L2D_PLAN_NO_PROBE)) {
        st = cached_sm_map(d.device, p->sm_domain);
        if (st != L2D_OK) {
            delete p;
            return st;
        }
        uint64_t ab = 0, as = 0;
        st = alloc_range(d.A, &ab, &as);
        if (st != L2D_OK) {
            delete p;
            return st;
        }
        const uint64_t lo_tab = A & ~(kPageBytes - 1);
        const uint64_t hi_tab = (A + span + kPageBytes - 1) & ~(kPageBytes - 1);
        const uint64_t lo = std::max(lo_tab, (ab + kPageBytes - 1) & ~(kPageBytes - 1));
        const uint64_t hi = std::min(hi_tab, ab + as);
        p->region_base = reinterpret_cast<const uint8_t *>(lo_tab);
        p->attr.assign((hi_tab - lo_tab) / kPageBytes, 0);
        if (hi > lo) {
            size_t np = 0;
            std::vector<int> attr_sub((hi - lo + kPageBytes - 1) / kPageBytes, 0);
            st = probe_addr_domains_impl(d.device, reinterpret_cast<const uint8_t *>(lo), hi - lo,
                                         p->sm_domain.data(), p->num_sm, &p->mask, attr_sub.data(), attr_sub.size(),
                                         &np, nullptr, nullptr, nullptr, 0, nullptr);
            if (st != L2D_OK) {
                delete p;
                return st;
            }
            std::copy(attr_sub.begin(), attr_sub.end(), p->attr.begin() + (lo - lo_tab) / kPageBytes);
        }
        p->has_domains = true;
    }
    if (p->has_domains) {
        for (int s = 0; s < p->num_sm; ++s) p->n_dom[p->sm_domain[s] & 1]++;
        if (p->n_dom[0] == 0 || p->n_dom[1] == 0) p->has_domains = false;
        p->gran_shift = lowest_bit_or(p->mask, kPageShift);
    }
    p->n_slots = p->num_sm;
    domain_census(*p);

    // One device block: slot table, attr bits, partials, counters, claims, control words.
    std::vector<int32_t> slot(kMaxSmid, -1);
    {
        int next[2] = {0, p->n_dom[0]};
        for (int s = 0; s < p->num_sm; ++s) {
            if (p->has_domains) slot[s] = next[p->sm_domain[s] & 1]++;
            else slot[s] = s;
        }
    }
    const size_t n_attr_words = std::max<size_t>(1, (p->attr.size() + 31) / 32);
    std::vector<uint32_t> attr_bits(n_attr_words, 0);
    for (size_t i = 0; i < p->attr.size(); ++i)
        if (p->attr[i] & 1) attr_bits[i / 32] |= 1u << (i % 32);
    const size_t R = static_cast<size_t>(std::max<int64_t>(p->rows_total, 1));
    size_t off = 0;
    const size_t o_slot = off;
    off = align256(off + kMaxSmid * sizeof(int32_t));
    const size_t o_attr = off;
    off = align256(off + n_attr_words * sizeof(uint32_t));
    const size_t o_ctl = off;
    off = align256(off + 4 * sizeof(unsigned long long));
    const size_t o_claim = off;
    off = align256(off + static_cast<size_t>(p->n_slots) * sizeof(unsigned long long));
    const size_t o_cnt = off;
    off = align256(off + R * sizeof(uint32_t));
    const size_t o_part = off;
    off = align256(off + 2 * R * sizeof(float));
    p->dev_bytes = off;
    cudaError_t e = cudaMalloc(&p->dev_block, off);
    if (e != cudaSuccess) {
        delete p;
        return set_error(L2D_ERR_CUDA, "plan scratch (%zu bytes): %s", off, cudaGetErrorString(e));
    }
    uint8_t *blk = static_cast<uint8_t *>(p->dev_block);
    p->d_sm_slot = reinterpret_cast<int32_t *>(blk + o_slot);
    p->d_attr_bits = reinterpret_cast<uint32_t *>(blk + o_attr);
    p->d_ctl = reinterpret_cast<unsigned long long *>(blk + o_ctl);
    p->d_claim = reinterpret_cast<unsigned long long *>(blk + o_claim);
    p->d_cnt = reinterpret_cast<uint32_t *>(blk + o_cnt);
    p->d_part = reinterpret_cast<float *>(blk + o_part);
    e = cudaMemset(p->dev_block, 0, off);
    if (e == cudaSuccess) e = cudaMemcpy(p->d_sm_slot, slot.data(), kMaxSmid * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(p->d_attr_bits, attr_bits.data(), n_attr_words * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(p->dev_block);
        delete p;
        return set_error(L2D_ERR_CUDA, "plan upload: %s", cudaGetErrorString(e));
    }
    *out = p;
    return L2D_OK;
}

int l2d_plan_destroy(l2d_plan *p) {
    clear_error();
    if (!p) return L2D_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    cudaError_t e = p->dev_block ? cudaFree(p->dev_block) : cudaSuccess;
    if (prev >= 0) cudaSetDevice(prev);
    delete p;
    if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "plan_destroy: %s", cudaGetErrorString(e));
    return L2D_OK;
}

int l2d_gemv(l2d_plan *p, const void *A, const void *x, void *y, int mode, void *stream) {
    if (!p) return set_error(L2D_ERR_INVALID, "null plan");
    if (A != p->desc.A) return set_error(L2D_ERR_INVALID, "A differs from the planned allocation");
    if (mode < L2D_MODE_OBLIVIOUS || mode > L2D_MODE_STREAM) return set_error(L2D_ERR_INVALID, "bad mode %d", mode);
    if (p->rows_total == 0) return L2D_OK;
    if (!x || !y) return set_error(L2D_ERR_INVALID, "null x or y");
    if (reinterpret_cast<uintptr_t>(x) & 15) return set_error(L2D_ERR_UNSUPPORTED, "x must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(y) & (p->eb_out - 1)) return set_error(L2D_ERR_INVALID, "y is misaligned");
    // With N == 0 every row is y = 0 and no window exists to split: the unsplit kernel writes it.
    const bool split = mode != L2D_MODE_STREAM && p->desc.N > 0;
    if (split && !p->has_domains)
        return set_error(L2D_ERR_UNSUPPORTED, "plan has no domain map: only L2D_MODE_STREAM is available");
    GemvArgs a;
    a.A = static_cast<const uint8_t *>(A);
    a.x = static_cast<const uint8_t *>(x);
    a.y = static_cast<uint8_t *>(y);
    a.M = p->desc.M;
    a.row_bytes = p->desc.N * p->eb_in;
    a.lda_bytes = p->desc.lda * p->eb_in;
    a.stride_a_bytes = p->desc.stride_a * p->eb_in;
    a.stride_x_bytes = p->desc.stride_x * p->eb_in;
    a.stride_y_elems = p->desc.stride_y;
    a.rows_total = p->rows_total;
    a.region_base = split ? p->region_base : p->stream_base;
    a.attr_bits = p->d_attr_bits;
    a.mask = p->mask;
    a.gran_shift = p->gran_shift;
    a.dom_kind = mode == L2D_MODE_OBLIVIOUS ? 1 : 0;
    a.flip = mode == L2D_MODE_SWAPPED ? 1 : 0;
    a.sm_slot = p->d_sm_slot;
    a.n_slots = p->n_slots;
    a.n_dom0 = p->n_dom[0];
    a.n_dom1 = p->n_dom[1];
    a.part = p->d_part;
    a.cnt = p->d_cnt;
    a.claim = p->d_claim;
    a.ctl = p->d_ctl;
    KernelFn k = pick_kernel(p->desc.dtype_in, p->desc.dtype_out, split);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != p->device) cudaSetDevice(p->device);
    k<<<p->n_slots, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    cudaError_t e = cudaGetLastError();
    if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return L2D_OK;
}

int l2d_plan_stats_get(l2d_plan *p, l2d_plan_stats *s) {
    clear_error();
    if (!p || !s) return set_error(L2D_ERR_INVALID, "null argument");
    std::memset(s, 0, sizeof *s);
    s->rows_total = p->rows_total;
    s->granule_shift = p->gran_shift;
    s->domain_bytes[0] = p->domain_bytes[0];
    s->domain_bytes[1] = p->domain_bytes[1];
    s->split_rows = p->split_rows;
    s->domain_sms[0] = p->n_dom[0];
    s->domain_sms[1] = p->n_dom[1];
    s->grid = p->n_slots;
    s->block = kThreads;
    s->scratch_bytes = p->dev_bytes;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    unsigned long long ctl[4] = {0, 0, 0, 0};
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(ctl, p->d_ctl, sizeof ctl, cudaMemcpyDeviceToHost);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "plan_stats: %s", cudaGetErrorString(e));
    s->calls = ctl[0];
    s->fallback_slots = ctl[2];
    return L2D_OK;
}

int l2d_plan_domain_map(const l2d_plan *p, int *sm_domain, int cap, int *num_sm, uint32_t *mask) {
    if (!p) return set_error(L2D_ERR_INVALID, "null plan");
    if (num_sm) *num_sm = p->num_sm;
    if (mask) *mask = p->mask;
    if (sm_domain) {
        if (cap < p->num_sm) return set_error(L2D_ERR_INVALID, "capacity %d < %d", cap, p->num_sm);
        for (int i = 0; i < p->num_sm; ++i) sm_domain[i] = p->has_domains ? p->sm_domain[i] : 0;
    }
    return L2D_OK;
}

}  // extern "C"
