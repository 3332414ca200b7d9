// L2-domain-aware GEMV for sm_100a (y = A.x, fp32 accumulation).
//
// Reference: applications/gemv/src/gemv_k1024_persistent_subwarp.cu:141-231.  The reference runs a
// persistent grid of one 512-thread CTA per SM; an SM of side s walks a host-built list of whole
// rows homed on side s, one warp per row (K = 1024 fp32 = one 4 KiB granule, so a row never
// crosses domains), float4 loads, shuffle reduction.
//
// This kernel keeps the persistent-grid / one-CTA-per-SM shape, rebuilt for Blackwell:
//  * Work is split into 1 KiB units (absolute address alignment), not rows: the BASELINE rows are
//    8-32 KiB and cross many 4 KiB domain granules.  A unit's domain is computed in the kernel from
//    the probed XOR mask and the per-2-MiB-page attr bits (the reference's predictor), 64 units per
//    warp ballot, so no row lists are read.  The SMs of domain d stream exactly the units homed in
//    d (AWARE), the other domain's (SWAPPED), or a pseudo-random half at the probed granule size
//    (OBLIVIOUS); STREAM takes every unit of its rows.
//  * Each warp runs a producer/consumer pipeline over its rows: the producer walks the units the
//    group streams and issues them as cp.async copies (2 x 16 bytes per lane) into a per-warp ring
//    of 12 x 1 KiB shared-memory slots; the consumer reads slot k while the next 11 units are in
//    flight, so loads never drain at row boundaries and no register holds in-flight data.  x is
//    staged once per CTA as fp32 in shared memory (swizzled so lanes read it without bank
//    conflicts); A pairs are widened exactly (bf16: a shift and a mask; fp16: cvt) and multiplied
//    with packed fma.rn.f32x2.
//  * Per row, each domain group produces one fp32 partial.  Both partials travel inside one packed
//    64-bit atomicAdd (each half holds ~bits(partial)): the group that sees the other half already
//    present adds part[0] + part[1] (commutative, so deterministic) and stores y.  No fence, no
//    second kernel.
//  * Rows are blocked per slot (one slot per SM) and interleaved over the CTA's warps.  Slots are
//    claimed with a per-call epoch: a CTA whose SM slot is already taken takes any unclaimed slot,
//    and the last CTA to finish processes slots nobody claimed, so every row is computed exactly
//    once whatever the block scheduler does.  Nothing in the kernel waits on another CTA.
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

constexpr int kUnitShift = 10;  // 1 KiB units: 32 bytes per lane
constexpr int kWarps = 12;
constexpr int kThreads = kWarps * 32;
constexpr int kRing = 12;       // units per warp ring; kRing - 1 are in flight while one is consumed
constexpr int kRowRing = 16;    // row descriptors per warp (power of two, >= kRing + 2)
constexpr int kSmemLimit = 227 * 1024;

struct GemvArgs {
    const uint8_t *A;
    const uint8_t *x;
    uint8_t *y;
    int64_t M;
    int64_t N;
    int64_t row_bytes;
    int64_t lda_bytes;
    int64_t stride_a_bytes;
    int64_t stride_x_bytes;
    int64_t stride_y_elems;
    int64_t rows_total;
    const uint8_t *region_base;   // 1 KiB aligned (2 MiB aligned when the attr table is used)
    const uint32_t *attr_bits;    // per 2 MiB page of the region, 32 pages per word
    uint32_t mask;
    int gran_shift;
    int dom_kind;                 // 0 = probed XOR model, 1 = hash of the granule index
    int flip;                     // 1 = swapped control
    int x_smem;                   // 1 = x staged as fp32 in shared memory, 0 = read from global
    int64_t x_stride_f32;         // floats between staged x vectors (multiple of 32)
    const int32_t *sm_slot;       // [kMaxSmid] slot of each SM, -1 = none
    int n_slots;
    int n_dom0;
    int n_dom1;
    int64_t spill_num;            // row r is a spill row iff (r*num mod den) + num >= den
    int64_t spill_den;            // (spill rows are taken whole by big_grp; num = 0: no spill rows)
    int big_grp;                  // the group with more SMs
    unsigned long long *pair;     // [rows_total] packed partial pair, zero between calls
    unsigned long long *claim;    // [n_slots] epoch of the last claim
    unsigned long long *ctl;      // [0] epoch, [1] CTAs done, [2] fallback claims
};

// ---- per-warp shared-memory ring --------------------------------------------------------------

struct RowDesc {           // one row of the warp's stream
    int64_t rs;            // region-relative byte offset of the row start
    int32_t row, b, i;     // global row, problem, row within the problem
    int32_t flags;         // bit 0: this group owns units of the row, bit 1: the other group does,
                           // bit 2: the row is split between the groups
    int32_t pad[2];
};

struct UnitMeta {          // one slot of the data ring
    int64_t unit;          // region-relative unit index
    int32_t tag;           // row descriptor index, -1 = no unit (end of the stream)
    int32_t pad;
};

struct WarpRing {
    uint8_t data[kRing][1 << kUnitShift];
    UnitMeta meta[kRing];
    RowDesc rows[kRowRing];
};

constexpr size_t kRingBytes = sizeof(WarpRing) * kWarps;

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

// Domain of the 1 KiB unit u (region-relative index) as seen by the split.
__device__ __forceinline__ int unit_dom(const GemvArgs &a, uint64_t u) {
    const uint64_t ua = u << kUnitShift;
    int d;
    if (a.dom_kind == 0) {
        const uint64_t page = ua >> kPageShift;
        const int attr = (__ldg(a.attr_bits + (page >> 5)) >> (page & 31)) & 1;
        d = (__popc(static_cast<uint32_t>(ua) & a.mask) & 1) ^ attr;
    } else {
        d = mix_granule(ua >> a.gran_shift) & 1;
    }
    return d ^ a.flip;
}

// ---- arithmetic: widen to fp32, packed fma.rn.f32x2 --------------------------------------------

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long x,
                                                    unsigned long long c) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(a), "l"(x));
    return c;
}

template <int DT> __device__ __forceinline__ unsigned long long widen2(uint32_t v);
template <> __device__ __forceinline__ unsigned long long widen2<L2D_BF16>(uint32_t v) {
    return (static_cast<unsigned long long>(v & 0xffff0000u) << 32) | (v << 16);  // exact
}
template <> __device__ __forceinline__ unsigned long long widen2<L2D_F16>(uint32_t v) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&v));  // exact
    return pack2(f.x, f.y);
}

template <int DT> __device__ __forceinline__ float elem(const uint8_t *p) {
    if (DT == L2D_F32) return *reinterpret_cast<const float *>(p);
    const uint16_t h = *reinterpret_cast<const uint16_t *>(p);
    if (DT == L2D_F16) return __half2float(__ushort_as_half(h));
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// Lane accumulators: four packed pairs (eight fp32 partial sums) plus a scalar for edge elements.
struct Acc {
    unsigned long long p0, p1, p2, p3;
    float edge;
    __device__ __forceinline__ void reset() {
        p0 = p1 = p2 = p3 = 0ull;
        edge = 0.f;
    }
    __device__ __forceinline__ float total() const {
        const float2 a = *reinterpret_cast<const float2 *>(&p0), b = *reinterpret_cast<const float2 *>(&p1);
        const float2 c = *reinterpret_cast<const float2 *>(&p2), d = *reinterpret_cast<const float2 *>(&p3);
        return ((a.x + a.y) + (b.x + b.y)) + ((c.x + c.y) + (d.x + d.y)) + edge;
    }
};

// Swizzled position of 16-byte chunk Q of a staged fp32 x vector: lane l reads the C chunks
// 4l/C*... of its unit with C = 2 (fp32 A) or 4 (fp16/bf16 A), so XOR-ing the low bits with
// (Q >> 3) spreads every 8-lane group over all eight 16-byte bank groups (no bank conflicts).
template <int C> __device__ __forceinline__ int64_t swz(int64_t q) { return q ^ ((q >> 3) & (C - 1)); }

// One unit (32 bytes of A per lane) times the matching x: `e0` is the row-relative index of the
// lane's first element.
template <int DT, bool XS>
__device__ __forceinline__ void unit_fma(Acc &acc, const uint4 a0, const uint4 a1, const uint8_t *xrow, int64_t e0) {
    if (XS) {
        const float4 *xs = reinterpret_cast<const float4 *>(xrow);
        if (DT == L2D_F32) {
            const int64_t q = e0 >> 2;  // 8 elements: chunks q, q+1
            const float4 x0 = xs[swz<2>(q)], x1 = xs[swz<2>(q + 1)];
            acc.p0 = ffma2(pack2(__uint_as_float(a0.x), __uint_as_float(a0.y)), pack2(x0.x, x0.y), acc.p0);
            acc.p1 = ffma2(pack2(__uint_as_float(a0.z), __uint_as_float(a0.w)), pack2(x0.z, x0.w), acc.p1);
            acc.p2 = ffma2(pack2(__uint_as_float(a1.x), __uint_as_float(a1.y)), pack2(x1.x, x1.y), acc.p2);
            acc.p3 = ffma2(pack2(__uint_as_float(a1.z), __uint_as_float(a1.w)), pack2(x1.z, x1.w), acc.p3);
        } else {
            const int64_t q = e0 >> 2;  // 16 elements: chunks q .. q+3
            const float4 x0 = xs[swz<4>(q)], x1 = xs[swz<4>(q + 1)], x2 = xs[swz<4>(q + 2)], x3 = xs[swz<4>(q + 3)];
            acc.p0 = ffma2(widen2<DT>(a0.x), pack2(x0.x, x0.y), acc.p0);
            acc.p1 = ffma2(widen2<DT>(a0.y), pack2(x0.z, x0.w), acc.p1);
            acc.p2 = ffma2(widen2<DT>(a0.z), pack2(x1.x, x1.y), acc.p2);
            acc.p3 = ffma2(widen2<DT>(a0.w), pack2(x1.z, x1.w), acc.p3);
            acc.p0 = ffma2(widen2<DT>(a1.x), pack2(x2.x, x2.y), acc.p0);
            acc.p1 = ffma2(widen2<DT>(a1.y), pack2(x2.z, x2.w), acc.p1);
            acc.p2 = ffma2(widen2<DT>(a1.z), pack2(x3.x, x3.y), acc.p2);
            acc.p3 = ffma2(widen2<DT>(a1.w), pack2(x3.z, x3.w), acc.p3);
        }
    } else {
        constexpr int eb = DT == L2D_F32 ? 4 : 2;
        const uint8_t *xp = xrow + e0 * eb;
        uint4 x0, x1;
        asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x0.x), "=r"(x0.y), "=r"(x0.z), "=r"(x0.w) : "l"(xp));
        asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
            : "=r"(x1.x), "=r"(x1.y), "=r"(x1.z), "=r"(x1.w)
            : "l"(xp + 16));
        if (DT == L2D_F32) {
            acc.p0 = ffma2((static_cast<unsigned long long>(a0.y) << 32) | a0.x,
                           (static_cast<unsigned long long>(x0.y) << 32) | x0.x, acc.p0);
            acc.p1 = ffma2((static_cast<unsigned long long>(a0.w) << 32) | a0.z,
                           (static_cast<unsigned long long>(x0.w) << 32) | x0.z, acc.p1);
            acc.p2 = ffma2((static_cast<unsigned long long>(a1.y) << 32) | a1.x,
                           (static_cast<unsigned long long>(x1.y) << 32) | x1.x, acc.p2);
            acc.p3 = ffma2((static_cast<unsigned long long>(a1.w) << 32) | a1.z,
                           (static_cast<unsigned long long>(x1.w) << 32) | x1.z, acc.p3);
        } else {
            acc.p0 = ffma2(widen2<DT>(a0.x), widen2<DT>(x0.x), acc.p0);
            acc.p1 = ffma2(widen2<DT>(a0.y), widen2<DT>(x0.y), acc.p1);
            acc.p2 = ffma2(widen2<DT>(a0.z), widen2<DT>(x0.z), acc.p2);
            acc.p3 = ffma2(widen2<DT>(a0.w), widen2<DT>(x0.w), acc.p3);
            acc.p0 = ffma2(widen2<DT>(a1.x), widen2<DT>(x1.x), acc.p0);
            acc.p1 = ffma2(widen2<DT>(a1.y), widen2<DT>(x1.y), acc.p1);
            acc.p2 = ffma2(widen2<DT>(a1.z), widen2<DT>(x1.z), acc.p2);
            acc.p3 = ffma2(widen2<DT>(a1.w), widen2<DT>(x1.w), acc.p3);
        }
    }
}

// x element e of a row (staged fp32, swizzled, or global in the input type).
template <int DT, bool XS> __device__ __forceinline__ float x_elem(const uint8_t *xrow, int64_t e) {
    if (XS) {
        constexpr int C = DT == L2D_F32 ? 2 : 4;
        return reinterpret_cast<const float *>(xrow)[swz<C>(e >> 2) * 4 + (e & 3)];
    }
    constexpr int eb = DT == L2D_F32 ? 4 : 2;
    return elem<DT>(xrow + e * eb);
}

template <int DT> __device__ __forceinline__ void store_out(uint8_t *y, float v);
template <> __device__ __forceinline__ void store_out<L2D_F32>(uint8_t *y, float v) { *reinterpret_cast<float *>(y) = v; }
template <> __device__ __forceinline__ void store_out<L2D_F16>(uint8_t *y, float v) {
    *reinterpret_cast<__half *>(y) = __float2half_rn(v);
}
template <> __device__ __forceinline__ void store_out<L2D_BF16>(uint8_t *y, float v) {
    *reinterpret_cast<__nv_bfloat16 *>(y) = __float2bfloat16_rn(v);
}

// Stages the x vectors of problems [b0, b0 + nb) as fp32, swizzled, x_stride_f32 floats apart.
template <int DT> __device__ __forceinline__ void stage_x(const GemvArgs &a, float *xs, int64_t b0, int64_t nb) {
    constexpr int C = DT == L2D_F32 ? 2 : 4;
    constexpr int eb = DT == L2D_F32 ? 4 : 2;
    const int64_t chunks = a.x_stride_f32 / 4;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *src = a.x + (b0 + b) * a.stride_x_bytes;
        float4 *dst = reinterpret_cast<float4 *>(xs + b * a.x_stride_f32);
        for (int64_t q = threadIdx.x; q < chunks; q += blockDim.x) {
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int64_t e = 4 * q + k;
                v[k] = e < a.N ? elem<DT>(src + e * eb) : 0.f;
            }
            dst[swz<C>(q)] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();
}

// ---- rows ------------------------------------------------------------------------------------

// Balance between unequal domain groups: a fraction num/den = (n_big - n_small)/(n_big + n_small) of
// the rows, spread evenly, is taken whole by the bigger group and skipped by the smaller one.  Row r
// is such a spill row iff floor((r+1) num/den) > floor(r num/den), i.e. iff (r num mod den) + num >=
// den.  A warp walks its rows with a fixed stride, so it carries (r num mod den), the problem index
// and the row within the problem incrementally: no division per row.
struct RowIter {  // rows_total < 2^31 (checked when the call is set up)
    int32_t row, b, i;
    int32_t phase;  // row * num mod den
    __device__ __forceinline__ void start(const GemvArgs &a, int32_t r) {
        const int32_t M = static_cast<int32_t>(a.M);
        row = r;
        b = r / M;
        i = r - b * M;
        phase = a.spill_num ? static_cast<int32_t>(static_cast<int64_t>(r) * a.spill_num % a.spill_den) : 0;
    }
    __device__ __forceinline__ void advance(const GemvArgs &a, int32_t stride, int32_t step_phase) {
        const int32_t M = static_cast<int32_t>(a.M);
        row += stride;
        i += stride;
        while (i >= M) {
            i -= M;
            ++b;
        }
        phase += step_phase;
        if (phase >= a.spill_den) phase -= static_cast<int32_t>(a.spill_den);
    }
    __device__ __forceinline__ bool spill(const GemvArgs &a) const {
        return a.spill_num != 0 && phase + a.spill_num >= a.spill_den;
    }
};

// A row whose pair atomic has been issued by lane 0 but whose returned value is not inspected
// yet; it is resolved at the warp's next publish, so the atomic's round trip overlaps with work.
struct Pending {
    unsigned long long old;
    uint8_t *yp;
    int32_t row;
    float sum;
    int grp;
    bool active;
};

template <int DT_OUT> __device__ __forceinline__ void resolve(const GemvArgs &a, Pending &p) {
    if (!p.active) return;
    p.active = false;
    const uint32_t other = static_cast<uint32_t>(p.old >> (32 * (p.grp ^ 1)));
    if (other != 0u) {
        store_out<DT_OUT>(p.yp, p.sum + __uint_as_float(~other));  // commutative: same bits either way
        a.pair[p.row] = 0ull;
    }
}

// Lane 0: the row's result.  A row owned by one group is stored directly.  Otherwise each group adds
// ~bits(partial) into its own 32-bit half of the row's pair word; ~bits is never 0 for a value
// arithmetic produces, so the group that finds the other half non-zero holds both partials and
// finishes the row (in resolve, at this warp's next publish).
template <int DT_OUT>
__device__ __forceinline__ void publish(const GemvArgs &a, Pending &pend, int32_t row, int32_t b, int32_t i, int grp,
                                        bool shared, float sum) {
    constexpr int eo = DT_OUT == L2D_F32 ? 4 : 2;
    uint8_t *yp = a.y + (static_cast<int64_t>(b) * a.stride_y_elems + i) * eo;
    if (!shared) {
        store_out<DT_OUT>(yp, sum);
        return;
    }
    resolve<DT_OUT>(a, pend);
    pend.old = atomicAdd(a.pair + row, static_cast<unsigned long long>(~__float_as_uint(sum)) << (32 * grp));
    pend.yp = yp;
    pend.row = row;
    pend.sum = sum;
    pend.grp = grp;
    pend.active = true;
}

// The edge units of a row (cut by its start or end, at most two) that this group owns, element by
// element into acc.edge.
template <int DT, bool XS>
__device__ __forceinline__ void row_edges(const GemvArgs &a, Acc &acc, uint64_t rs, const uint8_t *xrow, bool split,
                                          int grp, int lane) {
    constexpr int eb = DT == L2D_F32 ? 4 : 2;
    const uint64_t re = rs + static_cast<uint64_t>(a.row_bytes);
    const uint64_t ufirst = rs >> kUnitShift, ulast = (re - 1) >> kUnitShift;
    for (int k = 0; k < 2; ++k) {
        const uint64_t u = k == 0 ? ufirst : ulast;
        if (k == 1 && ulast == ufirst) break;
        const bool full = (u << kUnitShift) >= rs && ((u + 1) << kUnitShift) <= re;
        if (full || (split && unit_dom(a, u) != grp)) continue;
        const uint64_t p0 = (u << kUnitShift) + lane * 32;
        const uint64_t lo = p0 > rs ? p0 : rs, hi = p0 + 32 < re ? p0 + 32 : re;
        for (uint64_t o = lo; o < hi; o += eb)
            acc.edge = fmaf(elem<DT>(a.region_base + o), x_elem<DT, XS>(xrow, static_cast<int64_t>((o - rs) / eb)),
                            acc.edge);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The warp's producer: walks the warp's rows and, within each, the 1 KiB units this group streams
// (full units of its domain, or every full unit of an unsplit row), 64 units per ballot.
struct Producer {
    RowIter it;
    uint64_t rs, re, ub, uend, mask;
    int32_t tag, flags, next_tag;
    bool active, split;
};

template <int DT, int DT_OUT, bool XS, bool SPLIT>
struct Pipeline {
    const GemvArgs &a;
    WarpRing &W;
    const float *xs;   // staged x of problem xs_b0 (XS)
    int64_t xs_b0;
    int grp, lane, nwarps;
    int64_t r1;
    bool small_grp;
    int32_t step_phase;
    Producer P;
    Pending pend;

    __device__ __forceinline__ const uint8_t *xrow_of(int32_t b) const {
        if (XS) return reinterpret_cast<const uint8_t *>(xs + (b - xs_b0) * a.x_stride_f32);
        return a.x + static_cast<int64_t>(b) * a.stride_x_bytes;
    }

    __device__ __forceinline__ void block_mask() {
        const uint64_t ua = P.ub + lane, uc = P.ub + 32 + lane;
        const bool ina = ua < P.uend, inc = uc < P.uend;
        const bool fa = ina && (ua << kUnitShift) >= P.rs && ((ua + 1) << kUnitShift) <= P.re;
        const bool fc = inc && (uc << kUnitShift) >= P.rs && ((uc + 1) << kUnitShift) <= P.re;
        bool ma = ina, mc = inc;
        if (SPLIT && P.split) {
            ma = ina && unit_dom(a, ua) == grp;
            mc = inc && unit_dom(a, uc) == grp;
        }
        P.mask = static_cast<uint64_t>(__ballot_sync(0xffffffffu, ma && fa)) |
                 (static_cast<uint64_t>(__ballot_sync(0xffffffffu, mc && fc)) << 32);
        const bool mine = __any_sync(0xffffffffu, ma || mc);
        const bool other = __any_sync(0xffffffffu, (ina && !ma) || (inc && !mc));
        P.flags |= (mine ? 1 : 0) | (other ? 2 : 0);
    }

    __device__ __forceinline__ void setup_row() {
        const int64_t off = static_cast<int64_t>(P.it.b) * a.stride_a_bytes + static_cast<int64_t>(P.it.i) * a.lda_bytes;
        P.rs = static_cast<uint64_t>(a.A + off - a.region_base);
        P.re = P.rs + static_cast<uint64_t>(a.row_bytes);
        P.ub = P.rs >> kUnitShift;
        P.uend = (P.re + (1u << kUnitShift) - 1) >> kUnitShift;
        P.tag = -1;
        P.flags = (SPLIT && P.split) ? 4 : 0;
        P.mask = 0;
        if (P.ub < P.uend) block_mask();
    }

    // Moves the producer to its next row (skipping spill rows in the smaller group); false at the end.
    __device__ __forceinline__ bool next_row(bool first) {
        for (;;) {
            if (!first) P.it.advance(a, nwarps, step_phase);
            first = false;
            if (P.it.row >= r1) return false;
            const bool spill = SPLIT && P.it.spill(a);
            if (spill && small_grp) continue;
            P.split = SPLIT && !spill;
            setup_row();
            return true;
        }
    }

    // A row with no full unit of this group: its edge units (if any are ours) finish it here.
    __device__ __forceinline__ void finish_without_units() {
        if (a.row_bytes == 0) {  // N == 0: y = 0, written once
            if (lane == 0 && grp == 0) publish<DT_OUT>(a, pend, P.it.row, P.it.b, P.it.i, grp, false, 0.f);
            return;
        }
        if (!(P.flags & 1)) return;
        Acc acc;
        acc.reset();
        row_edges<DT, XS>(a, acc, P.rs, xrow_of(P.it.b), SPLIT && P.split, grp, lane);
        const float s = warp_sum(acc.total());
        if (lane == 0) publish<DT_OUT>(a, pend, P.it.row, P.it.b, P.it.i, grp, (P.flags & 6) == 6, s);
    }

    // Next unit of the stream into (*unit, *tag); false when the stream is over.
    __device__ __forceinline__ bool next_unit(uint64_t *unit, int32_t *tag) {
        for (;;) {
            if (!P.active) return false;
            if (P.mask) {
                const int bit = __ffsll(static_cast<long long>(P.mask)) - 1;
                P.mask &= P.mask - 1;
                if (P.tag < 0) {
                    P.tag = P.next_tag;
                    P.next_tag = (P.next_tag + 1) & (kRowRing - 1);
                    if (lane == 0) {
                        RowDesc &d = W.rows[P.tag];
                        d.rs = static_cast<int64_t>(P.rs);
                        d.row = P.it.row;
                        d.b = P.it.b;
                        d.i = P.it.i;
                        d.flags = P.flags;
                    }
                }
                *unit = P.ub + bit;
                *tag = P.tag;
                return true;
            }
            if (P.ub + 64 < P.uend) {
                P.ub += 64;
                block_mask();
                if (P.tag >= 0 && lane == 0) W.rows[P.tag].flags = P.flags;
                continue;
            }
            if (P.tag >= 0) {
                if (lane == 0) W.rows[P.tag].flags = P.flags;
            } else {
                finish_without_units();
            }
            P.active = next_row(false);
        }
    }

    // Issues the next unit's two 16-byte async copies into ring slot s (or marks the slot empty);
    // one commit group per slot keeps the group count aligned with the ring.
    __device__ __forceinline__ void issue(int s) {
        uint64_t unit;
        int32_t tag;
        if (next_unit(&unit, &tag)) {
            const uint8_t *src = a.region_base + (unit << kUnitShift) + lane * 32;
            uint8_t *dst = W.data[s] + lane * 32;
            cp_async16(dst, src);
            cp_async16(dst + 16, src + 16);
            if (lane == 0) {
                W.meta[s].unit = static_cast<int64_t>(unit);
                W.meta[s].tag = tag;
            }
        } else if (lane == 0) {
            W.meta[s].tag = -1;
        }
        cp_async_commit();
    }

    __device__ __forceinline__ void flush(int32_t ctag, Acc &acc, uint64_t crs, const uint8_t *cx) {
        const RowDesc &d = W.rows[ctag];
        const int32_t flags = d.flags;
        row_edges<DT, XS>(a, acc, crs, cx, (flags & 4) != 0, grp, lane);
        const float s = warp_sum(acc.total());
        if (lane == 0) publish<DT_OUT>(a, pend, d.row, d.b, d.i, grp, (flags & 6) == 6, s);
    }

    __device__ __forceinline__ void run(int64_t r0) {
        pend.active = false;
        P.next_tag = 0;
        P.active = false;
        if (r0 + (threadIdx.x >> 5) < r1) {
            P.it.start(a, static_cast<int32_t>(r0 + (threadIdx.x >> 5)));
            P.active = next_row(true);
        }
        for (int s = 0; s < kRing - 1; ++s) issue(s);
        int ps = kRing - 1, cs = 0;
        int32_t ctag = -1;
        uint64_t crs = 0;
        const uint8_t *cx = nullptr;
        Acc acc;
        acc.reset();
        for (;;) {
            issue(ps);
            ps = ps + 1 == kRing ? 0 : ps + 1;
            cp_async_wait<kRing - 1>();
            __syncwarp();
            const int32_t tag = W.meta[cs].tag;
            if (tag < 0) break;
            const int64_t unit = W.meta[cs].unit;
            if (tag != ctag) {
                if (ctag >= 0) {
                    flush(ctag, acc, crs, cx);
                    acc.reset();
                }
                ctag = tag;
                crs = static_cast<uint64_t>(W.rows[tag].rs);
                cx = xrow_of(W.rows[tag].b);
            }
            const uint4 *sp = reinterpret_cast<const uint4 *>(W.data[cs] + lane * 32);
            const uint4 a0 = sp[0], a1 = sp[1];
            constexpr int eb = DT == L2D_F32 ? 4 : 2;
            const int64_t e0 = (static_cast<int64_t>(unit << kUnitShift) + lane * 32 - static_cast<int64_t>(crs)) / eb;
            unit_fma<DT, XS>(acc, a0, a1, cx, e0);
            __syncwarp();
            cs = cs + 1 == kRing ? 0 : cs + 1;
        }
        cp_async_wait<0>();
        if (ctag >= 0) flush(ctag, acc, crs, cx);
        if (lane == 0) resolve<DT_OUT>(a, pend);
        __syncwarp();
    }
};

template <int DT_IN, int DT_OUT, bool SPLIT>
__device__ __forceinline__ void run_slot(const GemvArgs &a, int slot, int warp, int nwarps, int lane, uint8_t *smem) {
    int grp = 0, idx = slot, n_group = a.n_slots;
    if (SPLIT) {
        grp = slot >= a.n_dom0;
        idx = grp ? slot - a.n_dom0 : slot;
        n_group = grp ? a.n_dom1 : a.n_dom0;
    }
    const int64_t r0 = a.rows_total * idx / n_group;
    const int64_t r1 = a.rows_total * (idx + 1) / n_group;
    if (r0 >= r1) return;
    WarpRing *rings = reinterpret_cast<WarpRing *>(smem);
    float *xs = reinterpret_cast<float *>(smem + kRingBytes);
    const int64_t b0 = r0 / a.M;
    const int32_t step_phase =
        a.spill_num ? static_cast<int32_t>(static_cast<int64_t>(nwarps) * a.spill_num % a.spill_den) : 0;
    const bool small_grp = SPLIT && a.spill_num != 0 && grp != a.big_grp;
    if (a.x_smem) {
        stage_x<DT_IN>(a, xs, b0, (r1 - 1) / a.M - b0 + 1);
        Pipeline<DT_IN, DT_OUT, true, SPLIT> p{a, rings[warp], xs, b0, grp, lane, nwarps, r1, small_grp, step_phase};
        p.run(r0);
    } else {
        Pipeline<DT_IN, DT_OUT, false, SPLIT> p{a, rings[warp], xs, b0, grp, lane, nwarps, r1, small_grp, step_phase};
        p.run(r0);
    }
    __syncthreads();  // the staged x and the rings may be reused for the next slot
}

__device__ __forceinline__ unsigned long long ld_claim(const unsigned long long *p) {
    return *reinterpret_cast<const volatile unsigned long long *>(p);
}

// Warp-wide search for an unclaimed slot (epoch older than E): 32 slots are read per step and only
// candidates are tried with atomicMax.  Returns the slot won, or -1 when none is left.
__device__ __forceinline__ int warp_claim_any(const GemvArgs &a, unsigned long long E, int lane) {
    for (int base = 0; base < a.n_slots; base += 32) {
        const int t = base + lane;
        const bool cand = t < a.n_slots && ld_claim(a.claim + t) < E;
        uint32_t m = __ballot_sync(0xffffffffu, cand);
        while (m) {
            const int l = __ffs(m) - 1;
            m &= m - 1;
            int ok = 0;
            if (lane == l) ok = atomicMax(a.claim + t, E) < E;
            if (__shfl_sync(0xffffffffu, ok, l)) return base + l;
        }
    }
    return -1;
}

template <int DT_IN, int DT_OUT, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_slot;
    __shared__ int s_last;
    __shared__ int s_count;
    __shared__ int s_list[kMaxSmid];
    __shared__ unsigned long long s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    if (warp == 0) {
        const unsigned long long E = ld_claim(a.ctl) + 1ull;
        int got = -1;
        if (lane == 0) {
            const uint32_t sm = dev::smid();
            const int home = sm < static_cast<uint32_t>(kMaxSmid) ? a.sm_slot[sm] : -1;
            if (home >= 0 && atomicMax(a.claim + home, E) < E) got = home;
        }
        got = __shfl_sync(0xffffffffu, got, 0);
        if (got < 0) {  // this SM's slot is taken (two CTAs on one SM): any unclaimed slot will do
            got = warp_claim_any(a, E, lane);
            if (got >= 0 && lane == 0) atomicAdd(a.ctl + 2, 1ull);
        }
        if (lane == 0) {
            s_slot = got;
            s_epoch = E;
            s_count = 0;
        }
    }
    __syncthreads();
    if (s_slot >= 0) run_slot<DT_IN, DT_OUT, SPLIT>(a, s_slot, warp, nwarps, lane, smem);
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned long long done = atomicAdd(a.ctl + 1, 1ull);
        s_last = done == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    // Last CTA: slots whose SM never hosted a CTA of this launch, found by one parallel sweep.
    const unsigned long long E = s_epoch;
    for (int t = tid; t < a.n_slots; t += blockDim.x) {
        if (ld_claim(a.claim + t) < E && atomicMax(a.claim + t, E) < E) s_list[atomicAdd(&s_count, 1)] = t;
    }
    __syncthreads();
    const int n_left = s_count;
    if (tid == 0 && n_left) atomicAdd(a.ctl + 2, static_cast<unsigned long long>(n_left));
    for (int k = 0; k < n_left; ++k) {
        run_slot<DT_IN, DT_OUT, SPLIT>(a, s_list[k], warp, nwarps, lane, smem);
        __syncthreads();
    }
    if (tid == 0) {
        a.ctl[1] = 0ull;
        __threadfence();
        *reinterpret_cast<volatile unsigned long long *>(a.ctl) = E;
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

// The kernels' dynamic shared-memory limit is process-wide state of each kernel, so it is raised once
// per kernel and device to the device maximum (every launch then passes its own size) instead of
// per plan, where a later plan with a smaller size would break an earlier plan's launches.
int allow_max_smem(KernelFn k, int device) {
    static std::mutex mu;
    static std::vector<std::pair<KernelFn, int>> done;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : done)
        if (e.first == k && e.second == device) return L2D_OK;
    int optin = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    cudaFuncAttributes fa;
    L2D_CUDA_TRY(cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(k)));
    L2D_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      optin - static_cast<int>(fa.sharedSizeBytes)));
    done.emplace_back(k, device);
    return L2D_OK;
}

// Shared memory of one launch: the warp rings plus the staged x when it fits (else x is read from
// global memory and x_stride_f32 is 0).  nb = the most problems any slot's rows can span.
size_t launch_smem(int64_t N, int64_t nb, int64_t *x_stride_f32) {
    const int64_t stride = (N + 31) / 32 * 32;
    const size_t budget = static_cast<size_t>(kSmemLimit) - 8 * 1024;  // static shared memory + margin
    const size_t xbytes = static_cast<size_t>(stride * 4 * nb);
    if (N > 0 && kRingBytes + xbytes <= budget) {
        *x_stride_f32 = stride;
        return kRingBytes + xbytes;
    }
    *x_stride_f32 = 0;
    return kRingBytes;
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
    const uint8_t *stream_base = nullptr;  // 1 KiB aligned base for the unsplit kernel
    int gran_shift = l2d::kPageShift;
    int n_dom[2] = {0, 0};
    int n_slots = 0;
    int64_t domain_bytes[2] = {0, 0};
    int64_t split_rows = 0;
    void *dev_block = nullptr;
    size_t dev_bytes = 0;
    int32_t *d_sm_slot = nullptr;
    uint32_t *d_attr_bits = nullptr;
    unsigned long long *d_pair = nullptr;
    size_t smem_bytes = 0;    // dynamic shared memory of a launch (warp rings + staged x)
    int64_t x_stride_f32 = 0; // floats between staged x vectors (0 = x read from global memory)
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
        for (uint64_t w = s >> kUnitShift; w < (e + 1023) >> kUnitShift; ++w) {
            uint64_t wa = w << kUnitShift;
            int d = l2d::parity_domain(p.mask, wa, p.attr[wa >> kPageShift]);
            uint64_t lo = std::max(wa, s), hi = std::min(wa + 1024, e);
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
    if (d.M > 0 && d.batch > (int64_t(1) << 31) / std::max<int64_t>(d.M, 1) - 1)
        return set_error(L2D_ERR_INVALID, "batch * M must stay below 2^31 rows");
    const int eb = elem_bytes(d.dtype_in);
    if (((d.lda * eb) & 15) || (d.batch > 1 && (((d.stride_a * eb) & 15) || ((d.stride_x * eb) & 15))))
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
    p->stream_base = reinterpret_cast<const uint8_t *>(A & ~uint64_t(1023));
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
    const size_t o_pair = off;
    off = align256(off + R * sizeof(unsigned long long));
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
    p->d_pair = reinterpret_cast<unsigned long long *>(blk + o_pair);
    e = cudaMemset(p->dev_block, 0, off);
    if (e == cudaSuccess) e = cudaMemcpy(p->d_sm_slot, slot.data(), kMaxSmid * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(p->d_attr_bits, attr_bits.data(), n_attr_words * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(p->dev_block);
        delete p;
        return set_error(L2D_ERR_CUDA, "plan upload: %s", cudaGetErrorString(e));
    }
    // Shared memory: the warp rings plus x staged as fp32 when it fits.  Every slot gets at most
    // R/n_min + 1 contiguous rows, and k contiguous rows touch at most ceil(k / M) + 1 problems.
    {
        int n_min = p->n_slots;
        if (p->has_domains) n_min = std::min({n_min, p->n_dom[0], p->n_dom[1]});
        const int64_t max_rows = p->rows_total / std::max(n_min, 1) + 2;
        const int64_t max_nb = std::min<int64_t>(d.batch, (max_rows + std::max<int64_t>(d.M, 1) - 1) /
                                                              std::max<int64_t>(d.M, 1) + 1);
        p->smem_bytes = launch_smem(d.N, max_nb, &p->x_stride_f32);
        for (bool split : {false, true}) {
            const int fe = allow_max_smem(pick_kernel(d.dtype_in, d.dtype_out, split), d.device);
            if (fe != L2D_OK) {
                cudaFree(p->dev_block);
                delete p;
                return fe;
            }
        }
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
    a.N = p->desc.N;
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
    a.pair = p->d_pair;
    a.x_smem = p->x_stride_f32 > 0;
    a.x_stride_f32 = p->x_stride_f32;
    // Balance between unequal domain groups: with n_small < n_big SMs, the bigger group also takes a
    // fraction (n_big - n_small)/(n_big + n_small) of the rows whole, spread evenly, so every SM
    // streams the same bytes.  The swapped control stays pure (no spill rows).
    a.big_grp = p->n_dom[1] > p->n_dom[0] ? 1 : 0;
    a.spill_num = 0;
    a.spill_den = 1;
    if (split && mode != L2D_MODE_SWAPPED && p->n_dom[0] != p->n_dom[1] && p->n_dom[0] > 0 && p->n_dom[1] > 0) {
        a.spill_num = std::abs(p->n_dom[1] - p->n_dom[0]);
        a.spill_den = p->n_dom[0] + p->n_dom[1];
    }
    a.claim = p->d_claim;
    a.ctl = p->d_ctl;
    KernelFn k = pick_kernel(p->desc.dtype_in, p->desc.dtype_out, split);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != p->device) cudaSetDevice(p->device);
    k<<<p->n_slots, kThreads, p->smem_bytes, static_cast<cudaStream_t>(stream)>>>(a);
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

// ---------------------------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot call cudaMalloc when they need a GEMV: a serving runtime that reserves nearly
// all HBM for its own pools at start-up and forbids later allocations, code running between
// cudaStreamBeginCapture and cudaStreamEndCapture (a cudaMalloc there breaks the capture), or a
// latency-critical path that must not enter the allocator.  l2d_gemv_noalloc runs the same kernel
// as l2d_gemv without a plan: its scratch (control words, slot claims, the SM->slot table, the
// attr bits and one pair word per row) lives in the file-scope array below, which every GPU that
// loads this library holds until the process exits.  Limits: L2D_NOALLOC_MAX_ROWS rows over all
// problems, L2D_NOALLOC_MAX_PAGES 2 MiB pages of A.  Every call shares the array and leaves its
// contents for the next call (the pair words return to zero when a call completes), so calls
// that overlap on the GPU (other streams, other threads) race and must be serialised by the
// caller.
// ---------------------------------------------------------------------------------------------

namespace l2d {
namespace noalloc {

constexpr size_t kCtlOff = 0;
constexpr size_t kClaimOff = 256;
constexpr size_t kSlotOff = kClaimOff + kMaxSmid * sizeof(unsigned long long);
constexpr size_t kAttrOff = kSlotOff + kMaxSmid * sizeof(int32_t);
constexpr size_t kPairOff = kAttrOff + (L2D_NOALLOC_MAX_PAGES / 32) * sizeof(uint32_t);
constexpr size_t kBytes = kPairOff + static_cast<size_t>(L2D_NOALLOC_MAX_ROWS) * sizeof(unsigned long long);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kBytes];

std::mutex g_mu;
uint8_t *g_ptr[kMaxDevices] = {nullptr};

// First call on a device: the device address of g_scratch (host code may not use the symbol
// itself as a pointer) and one clear of the whole array.  Runs with `device` current.
int setup(int device, uint8_t **out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ptr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess || !p)
            return set_error(L2D_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        e = cudaMemset(p, 0, kBytes);
        if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "clearing the static scratch: %s", cudaGetErrorString(e));
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "clearing the static scratch: %s", cudaGetErrorString(e));
        g_ptr[device] = static_cast<uint8_t *>(p);
    }
    *out = g_ptr[device];
    return L2D_OK;
}

}  // namespace noalloc
}  // namespace l2d

extern "C" int l2d_gemv_noalloc(const l2d_gemv_desc *desc_in, const l2d_domain_map *map, const void *x, void *y,
                                int mode, void *stream) {
    using namespace l2d;
    clear_error();
    if (!desc_in) return set_error(L2D_ERR_INVALID, "gemv_noalloc: null descriptor");
    l2d_gemv_desc d = *desc_in;
    if (d.M < 0 || d.N < 0 || !valid_dtype(d.dtype_in) || !valid_dtype(d.dtype_out))
        return set_error(L2D_ERR_INVALID, "gemv_noalloc: bad shape or dtype");
    if (mode < L2D_MODE_OBLIVIOUS || mode > L2D_MODE_STREAM) return set_error(L2D_ERR_INVALID, "bad mode %d", mode);
    if (d.lda == 0) d.lda = d.N;
    if (d.batch <= 0) d.batch = 1;
    if (d.stride_a == 0) d.stride_a = d.M * d.lda;
    if (d.stride_x == 0) d.stride_x = d.N;
    if (d.stride_y == 0) d.stride_y = d.M;
    if (d.lda < d.N || (d.batch > 1 && (d.stride_a < d.M * d.lda || d.stride_x < d.N || d.stride_y < d.M)))
        return set_error(L2D_ERR_INVALID, "gemv_noalloc: lda or strides too small");
    const int64_t R = d.batch * d.M;
    if (R > L2D_NOALLOC_MAX_ROWS)
        return set_error(L2D_ERR_INVALID, "gemv_noalloc: %lld rows exceed the allocation-free limit of %d rows",
                         (long long)R, L2D_NOALLOC_MAX_ROWS);
    if (R == 0) return L2D_OK;
    const int eb = elem_bytes(d.dtype_in), eo = elem_bytes(d.dtype_out);
    if (((d.lda * eb) & 15) || (d.batch > 1 && (((d.stride_a * eb) & 15) || ((d.stride_x * eb) & 15))))
        return set_error(L2D_ERR_UNSUPPORTED, "lda, stride_a and stride_x must be multiples of 16 bytes");
    if ((reinterpret_cast<uintptr_t>(d.A) & 15) || (reinterpret_cast<uintptr_t>(x) & 15))
        return set_error(L2D_ERR_UNSUPPORTED, "A and x must be 16-byte aligned");
    if (!d.A || !x || !y || (reinterpret_cast<uintptr_t>(y) & (eo - 1)))
        return set_error(L2D_ERR_INVALID, "null or misaligned A, x or y");
    const bool split = mode != L2D_MODE_STREAM && d.N > 0;
    if (split && (!map || !map->sm_domain || !map->attr))
        return set_error(L2D_ERR_UNSUPPORTED, "gemv_noalloc: modes other than STREAM need a domain map");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (d.device < 0 || d.device >= ndev || d.device >= noalloc::kMaxDevices)
        return set_error(L2D_ERR_INVALID, "device %d out of range", d.device);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != d.device) L2D_CUDA_TRY(cudaSetDevice(d.device));
    struct Restore {
        int prev, dev;
        ~Restore() {
            if (prev >= 0 && prev != dev) cudaSetDevice(prev);
        }
    } restore{prev, d.device};
    int num_sm = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&num_sm, cudaDevAttrMultiProcessorCount, d.device));
    uint8_t *scratch = nullptr;
    int st = noalloc::setup(d.device, &scratch);
    if (st != L2D_OK) return st;

    // Host tables on the stack: SM -> slot and the attr bits of the pages A's rows touch.
    const uint64_t A = reinterpret_cast<uint64_t>(d.A);
    const uint64_t span = static_cast<uint64_t>(((R - 1) / d.M * d.stride_a + (R - 1) % d.M * d.lda + d.N) * eb);
    int32_t slot[kMaxSmid];
    uint32_t attr_bits[L2D_NOALLOC_MAX_PAGES / 32];
    int n_dom[2] = {0, 0};
    size_t attr_words = 1;
    attr_bits[0] = 0;
    const uint8_t *region = reinterpret_cast<const uint8_t *>(A & ~uint64_t(1023));
    uint32_t mask = 0;
    int gran_shift = kPageShift;
    for (int s = 0; s < kMaxSmid; ++s) slot[s] = -1;
    if (split) {
        if (map->num_sm != num_sm) return set_error(L2D_ERR_INVALID, "domain map has %d SMs, device has %d",
                                                    map->num_sm, num_sm);
        const uint64_t base = reinterpret_cast<uint64_t>(map->base);
        if (base % kPageBytes || base > A || A + span > base + map->num_pages * kPageBytes)
            return set_error(L2D_ERR_INVALID, "domain map region does not cover A");
        if (map->num_pages > static_cast<size_t>(L2D_NOALLOC_MAX_PAGES))
            return set_error(L2D_ERR_INVALID, "gemv_noalloc: %zu pages exceed the limit of %d", map->num_pages,
                             L2D_NOALLOC_MAX_PAGES);
        int next[2] = {0, 0};
        for (int s = 0; s < num_sm; ++s) n_dom[map->sm_domain[s] & 1]++;
        if (n_dom[0] == 0 || n_dom[1] == 0) return set_error(L2D_ERR_INVALID, "domain map has an empty domain");
        next[1] = n_dom[0];
        for (int s = 0; s < num_sm; ++s) slot[s] = next[map->sm_domain[s] & 1]++;
        attr_words = (map->num_pages + 31) / 32;
        for (size_t w = 0; w < attr_words; ++w) attr_bits[w] = 0;
        for (size_t i = 0; i < map->num_pages; ++i)
            if (map->attr[i] & 1) attr_bits[i / 32] |= 1u << (i % 32);
        region = reinterpret_cast<const uint8_t *>(base);
        mask = map->mask;
        gran_shift = lowest_bit_or(mask, kPageShift);
    } else {
        for (int s = 0; s < num_sm && s < kMaxSmid; ++s) slot[s] = s;
    }
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    L2D_CUDA_TRY(cudaMemcpyAsync(scratch + noalloc::kSlotOff, slot, sizeof slot, cudaMemcpyHostToDevice, cs));
    L2D_CUDA_TRY(cudaMemcpyAsync(scratch + noalloc::kAttrOff, attr_bits, attr_words * sizeof(uint32_t),
                                 cudaMemcpyHostToDevice, cs));

    GemvArgs a;
    a.A = static_cast<const uint8_t *>(d.A);
    a.x = static_cast<const uint8_t *>(x);
    a.y = static_cast<uint8_t *>(y);
    a.M = d.M;
    a.N = d.N;
    a.row_bytes = d.N * eb;
    a.lda_bytes = d.lda * eb;
    a.stride_a_bytes = d.stride_a * eb;
    a.stride_x_bytes = d.stride_x * eb;
    a.stride_y_elems = d.stride_y;
    a.rows_total = R;
    a.region_base = region;
    a.attr_bits = reinterpret_cast<const uint32_t *>(scratch + noalloc::kAttrOff);
    a.mask = mask;
    a.gran_shift = gran_shift;
    a.dom_kind = mode == L2D_MODE_OBLIVIOUS ? 1 : 0;
    a.flip = mode == L2D_MODE_SWAPPED ? 1 : 0;
    a.sm_slot = reinterpret_cast<const int32_t *>(scratch + noalloc::kSlotOff);
    a.n_slots = num_sm;
    a.n_dom0 = n_dom[0];
    a.n_dom1 = n_dom[1];
    a.pair = reinterpret_cast<unsigned long long *>(scratch + noalloc::kPairOff);
    a.claim = reinterpret_cast<unsigned long long *>(scratch + noalloc::kClaimOff);
    a.ctl = reinterpret_cast<unsigned long long *>(scratch + noalloc::kCtlOff);
    a.big_grp = n_dom[1] > n_dom[0] ? 1 : 0;
    a.spill_num = 0;
    a.spill_den = 1;
    if (split && mode != L2D_MODE_SWAPPED && n_dom[0] != n_dom[1]) {
        a.spill_num = std::abs(n_dom[1] - n_dom[0]);
        a.spill_den = n_dom[0] + n_dom[1];
    }
    // Shared memory, sized as l2d_plan_create sizes it.
    int n_min = num_sm;
    if (split) n_min = std::min({n_min, n_dom[0], n_dom[1]});
    const int64_t max_rows = R / std::max(n_min, 1) + 2;
    const int64_t max_nb = std::min<int64_t>(d.batch, (max_rows + std::max<int64_t>(d.M, 1) - 1) /
                                                          std::max<int64_t>(d.M, 1) + 1);
    int64_t x_stride = 0;
    const size_t smem = launch_smem(d.N, max_nb, &x_stride);
    a.x_smem = x_stride > 0;
    a.x_stride_f32 = x_stride;
    KernelFn k = pick_kernel(d.dtype_in, d.dtype_out, split);
    st = allow_max_smem(k, d.device);
    if (st != L2D_OK) return st;
    k<<<num_sm, kThreads, smem, cs>>>(a);
    L2D_CUDA_TRY(cudaGetLastError());
    return L2D_OK;
}
