// Blackwell L2-domain probes.
//
// P1 (SM -> domain) replaces get_map_smid2side (utility/latopt.cuh:487-562, utility/get_smid2side.cu).
// The reference walks the SMs one at a time: SM 0 primes 16 lines of SM t's private slice,
// SM t times them, and a latency spread above 100 cycles marks the far side; waits are unbounded.
// Here one cooperative launch places exactly one CTA on every SM, the leader primes every
// target's private lines at once, all targets time their lines in parallel, and the leader then
// re-times every line.  The host (l2d_analyze_sm) classifies with a 2-means split and handles
// both cache behaviours a two-die L2 can have (far lines cached near after use, or not).
//
// P2 (address -> domain) replaces get_map_memory_attr (latopt.cuh:683-814, utility/get_mask.cu).
// Domain-1 SMs prime lines, a grid-wide (bounded) barrier follows, then domain-0 SMs time each
// line once.  Lines at 2^b offsets fit the XOR mask, random lines validate it, and every line
// votes for its 2 MiB page's attr bit (l2d_analyze_addr).  All lines of all pages are measured in
// one launch instead of one cross-SM handshake per page.
//
// Every wait is bounded by %globaltimer; a timeout sets a status bit and the kernel returns.
#include "l2d_device.cuh"
#include "l2d_internal.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <random>
#include <unordered_set>
#include <vector>

namespace l2d {

enum : uint32_t { kStatusTimeoutFlag = 1u, kStatusTimeoutDone = 2u, kStatusTicket = 4u, kStatusTimeoutPrime = 8u };

struct SmProbeArgs {
    const uint8_t *ws;
    const uint64_t *line_off;  // [grid * L]
    const uint64_t *warm_off;  // [grid * L] a line of the same 2 MiB page that is never probed
    uint32_t *smid_of;         // [grid]
    uint32_t *lat_t1;          // [grid * L] target, first access
    uint32_t *lat_t2;          // [grid * L] target, second access
    uint32_t *lat_l;           // [grid * L] leader, after all targets
    uint32_t *ctl;             // [0] primed flag, [1] targets done, [2] status bits
    uint64_t *sink;
    int L;
    uint64_t timeout_ns;
};

__global__ void k_probe_sm_domains(SmProbeArgs a) {
    if (threadIdx.x != 0) return;
    __shared__ volatile uint64_t sink;
    const uint64_t deadline = dev::globaltimer_ns() + a.timeout_ns;
    const int G = gridDim.x;
    const int c = blockIdx.x;
    a.smid_of[c] = dev::smid();
    sink = 0;
    if (c == 0) {
        uint64_t acc = 0;
        for (int t = 1; t < G; ++t)
            for (int j = 0; j < a.L; ++j) acc ^= dev::ld_cg_u64(a.ws + a.line_off[static_cast<size_t>(t) * a.L + j]);
        sink = acc;
        __threadfence();
        dev::st_release_u32(&a.ctl[0], 1u);
        if (!dev::wait_at_least(&a.ctl[1], static_cast<uint32_t>(G - 1), deadline)) {
            atomicOr(&a.ctl[2], kStatusTimeoutDone);
            return;
        }
        for (int t = 1; t < G; ++t) {
            for (int j = 0; j < a.L; ++j) {
                size_t i = static_cast<size_t>(t) * a.L + j;
                sink = dev::ld_cg_u64(a.ws + a.warm_off[i]);
                a.lat_l[i] = dev::timed_load(a.ws + a.line_off[i], &sink);
            }
        }
        a.sink[0] = sink;
        return;
    }
    if (!dev::wait_at_least(&a.ctl[0], 1u, deadline)) {
        atomicOr(&a.ctl[2], kStatusTimeoutFlag);
        atomicAdd(&a.ctl[1], 1u);
        return;
    }
    const size_t row = static_cast<size_t>(c) * a.L;
    for (int j = 0; j < a.L; ++j) {
        sink = dev::ld_cg_u64(a.ws + a.warm_off[row + j]);
        a.lat_t1[row + j] = dev::timed_load(a.ws + a.line_off[row + j], &sink);
    }
    for (int j = 0; j < a.L; ++j) a.lat_t2[row + j] = dev::timed_load(a.ws + a.line_off[row + j], &sink);
    a.sink[c] = sink;
    __threadfence();
    atomicAdd(&a.ctl[1], 1u);
}

struct AddrProbeArgs {
    const uint8_t *base;
    const uint64_t *off;      // [n] line offsets from base
    const uint64_t *warm;     // [n] same-page warm-up line offsets
    uint32_t n;
    const int *sm_domain;     // [kMaxSmid], -1 = not in the map
    int n_dom[2];             // SMs per domain in the map
    uint32_t *lat;            // [n]
    uint32_t *ctl;            // [0] primers done, [1] ticket d0, [2] ticket d1, [3] status
    uint64_t *sink;
    uint64_t timeout_ns;
};

__global__ void k_probe_addr_domains(AddrProbeArgs a) {
    if (threadIdx.x != 0) return;
    __shared__ volatile uint64_t sink;
    const uint64_t deadline = dev::globaltimer_ns() + a.timeout_ns;
    const uint32_t s = dev::smid();
    const int d = s < static_cast<uint32_t>(kMaxSmid) ? a.sm_domain[s] : -1;
    sink = 0;
    if (d == 1) {
        uint32_t i = atomicAdd(&a.ctl[2], 1u);
        if (i >= static_cast<uint32_t>(a.n_dom[1])) {
            atomicOr(&a.ctl[3], kStatusTicket);
            return;
        }
        uint64_t acc = 0;
        for (uint32_t j = i; j < a.n; j += a.n_dom[1]) acc ^= dev::ld_cg_u64(a.base + a.off[j]);
        sink = acc;
        a.sink[blockIdx.x] = sink;
        __threadfence();
        atomicAdd(&a.ctl[0], 1u);
    } else if (d == 0) {
        uint32_t i = atomicAdd(&a.ctl[1], 1u);
        if (i >= static_cast<uint32_t>(a.n_dom[0])) {
            atomicOr(&a.ctl[3], kStatusTicket);
            return;
        }
        if (!dev::wait_at_least(&a.ctl[0], static_cast<uint32_t>(a.n_dom[1]), deadline)) {
            atomicOr(&a.ctl[3], kStatusTimeoutPrime);
            return;
        }
        for (uint32_t j = i; j < a.n; j += a.n_dom[0]) {
            sink = dev::ld_cg_u64(a.base + a.warm[j]);
            a.lat[j] = dev::timed_load(a.base + a.off[j], &sink);
        }
        a.sink[blockIdx.x] = sink;
    }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

struct DevBuf {
    void *p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    cudaError_t alloc(size_t bytes) { return cudaMalloc(&p, bytes); }
    template <typename T> T *as() const { return static_cast<T *>(p); }
};

uint64_t timeout_ns_of(const l2d_probe_opts *o) {
    uint32_t ms = (o && o->timeout_ms) ? o->timeout_ms : 1000u;
    return static_cast<uint64_t>(ms) * 1000000ull;
}

// Dynamic shared memory that admits only one probe CTA per SM (more than half the SM's pool).
int one_cta_per_sm_smem(int device, int *smem) {
    int per_sm = 0, per_block = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device));
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&per_block, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    int want = per_sm / 2 + 1024;
    if (want > per_block) want = per_block;
    *smem = want;
    return L2D_OK;
}

// Writes a buffer of twice the L2 size so no probe line is left in either L2 half.
int flush_l2(int device, cudaStream_t st) {
    int l2 = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device));
    DevBuf b;
    L2D_CUDA_TRY(b.alloc(static_cast<size_t>(l2) * 2));
    L2D_CUDA_TRY(cudaMemsetAsync(b.p, 0x5a, static_cast<size_t>(l2) * 2, st));
    L2D_CUDA_TRY(cudaStreamSynchronize(st));
    return L2D_OK;
}

template <typename K, typename A>
int launch_one_per_sm(K kernel, A &args, int grid, int device, float *ms) {
    int smem = 0;
    int st = one_cta_per_sm_smem(device, &smem);
    if (st != L2D_OK) return st;
    L2D_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int per_sm = 0;
    L2D_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32, smem));
    if (per_sm != 1)
        return set_error(L2D_ERR_PROBE_COVERAGE, "probe kernel fits %d CTAs per SM, expected exactly 1", per_sm);
    cudaEvent_t e0, e1;
    L2D_CUDA_TRY(cudaEventCreate(&e0));
    L2D_CUDA_TRY(cudaEventCreate(&e1));
    void *kargs[] = {&args};
    cudaEventRecord(e0, 0);
    cudaError_t err = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(kernel), dim3(grid), dim3(32), kargs,
                                                  static_cast<size_t>(smem), 0);
    cudaEventRecord(e1, 0);
    cudaError_t serr = cudaEventSynchronize(e1);
    float t = 0;
    cudaEventElapsedTime(&t, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (ms) *ms = t;
    if (err != cudaSuccess)
        return set_error(L2D_ERR_CUDA, "cooperative probe launch: %s", cudaGetErrorString(err));
    if (serr != cudaSuccess) return set_error(L2D_ERR_CUDA, "probe kernel: %s", cudaGetErrorString(serr));
    return L2D_OK;
}

}  // namespace

int probe_sm_domains_impl(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts,
                          l2d_sm_probe_report *report, uint32_t *raw, size_t raw_cap, size_t *raw_len) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", device);
    DeviceGuard guard(device);
    int G = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, device));
    if (num_sm) *num_sm = G;
    if (!map) return L2D_OK;
    if (cap < G) return set_error(L2D_ERR_INVALID, "map capacity %d < %d SMs", cap, G);
    const int L = (opts && opts->lines_per_sm) ? static_cast<int>(opts->lines_per_sm) : 48;
    if (L < 8 || L > 4096) return set_error(L2D_ERR_INVALID, "lines_per_sm must be in [8, 4096]");

    // Workspace: one 2 MiB page per SM, zero-filled so every page is backed.
    const size_t ws_bytes = static_cast<size_t>(G) * kPageBytes;
    DevBuf ws_raw;
    L2D_CUDA_TRY(ws_raw.alloc(ws_bytes + kPageBytes));
    uintptr_t ws_addr = (reinterpret_cast<uintptr_t>(ws_raw.p) + kPageBytes - 1) & ~(uintptr_t)(kPageBytes - 1);
    L2D_CUDA_TRY(cudaMemset(ws_raw.p, 0, ws_bytes + kPageBytes));

    // Private random lines for every CTA, spread over the whole workspace so that each CTA sees
    // lines of many pages (and both domains) whatever the address hash is.
    const size_t n = static_cast<size_t>(G) * L;
    std::vector<uint64_t> off(n), warm(n);
    std::mt19937_64 rng(0x5eed1234abcdull);
    std::unordered_set<uint64_t> used;
    const uint64_t lines_total = ws_bytes / 128;
    for (size_t i = 0; i < n; ++i) {
        uint64_t o;
        do {
            o = (rng() % lines_total) * 128;
        } while ((o & (kPageBytes - 1)) == kPageBytes - 128 || !used.insert(o).second);
        off[i] = o;
        warm[i] = (o & ~(kPageBytes - 1)) + kPageBytes - 128;
    }
    DevBuf d_off, d_warm, d_smid, d_t1, d_t2, d_l, d_ctl, d_sink;
    L2D_CUDA_TRY(d_off.alloc(n * 8));
    L2D_CUDA_TRY(d_warm.alloc(n * 8));
    L2D_CUDA_TRY(d_smid.alloc(G * 4));
    L2D_CUDA_TRY(d_t1.alloc(n * 4));
    L2D_CUDA_TRY(d_t2.alloc(n * 4));
    L2D_CUDA_TRY(d_l.alloc(n * 4));
    L2D_CUDA_TRY(d_ctl.alloc(16));
    L2D_CUDA_TRY(d_sink.alloc(static_cast<size_t>(G) * 8));
    L2D_CUDA_TRY(cudaMemcpy(d_off.p, off.data(), n * 8, cudaMemcpyHostToDevice));
    L2D_CUDA_TRY(cudaMemcpy(d_warm.p, warm.data(), n * 8, cudaMemcpyHostToDevice));
    L2D_CUDA_TRY(cudaMemset(d_t1.p, 0xff, n * 4));
    L2D_CUDA_TRY(cudaMemset(d_t2.p, 0xff, n * 4));
    L2D_CUDA_TRY(cudaMemset(d_l.p, 0xff, n * 4));
    L2D_CUDA_TRY(cudaMemset(d_ctl.p, 0, 16));
    L2D_CUDA_TRY(cudaMemset(d_smid.p, 0xff, G * 4));
    int st = flush_l2(device, 0);
    if (st != L2D_OK) return st;

    SmProbeArgs a;
    a.ws = reinterpret_cast<const uint8_t *>(ws_addr);
    a.line_off = d_off.as<uint64_t>();
    a.warm_off = d_warm.as<uint64_t>();
    a.smid_of = d_smid.as<uint32_t>();
    a.lat_t1 = d_t1.as<uint32_t>();
    a.lat_t2 = d_t2.as<uint32_t>();
    a.lat_l = d_l.as<uint32_t>();
    a.ctl = d_ctl.as<uint32_t>();
    a.sink = d_sink.as<uint64_t>();
    a.L = L;
    a.timeout_ns = timeout_ns_of(opts);
    float ms = 0;
    st = launch_one_per_sm(k_probe_sm_domains, a, G, device, &ms);
    if (st != L2D_OK) return st;

    std::vector<uint32_t> smid(G), t1(n), t2(n), ll(n), ctl(4);
    L2D_CUDA_TRY(cudaMemcpy(smid.data(), d_smid.p, G * 4, cudaMemcpyDeviceToHost));
    L2D_CUDA_TRY(cudaMemcpy(t1.data(), d_t1.p, n * 4, cudaMemcpyDeviceToHost));
    L2D_CUDA_TRY(cudaMemcpy(t2.data(), d_t2.p, n * 4, cudaMemcpyDeviceToHost));
    L2D_CUDA_TRY(cudaMemcpy(ll.data(), d_l.p, n * 4, cudaMemcpyDeviceToHost));
    L2D_CUDA_TRY(cudaMemcpy(ctl.data(), d_ctl.p, 16, cudaMemcpyDeviceToHost));
    size_t need = G + 3 * n;
    if (raw_len) *raw_len = need;
    if (raw && raw_cap >= need) {
        std::copy(smid.begin(), smid.end(), raw);
        std::copy(t1.begin(), t1.end(), raw + G);
        std::copy(t2.begin(), t2.end(), raw + G + n);
        std::copy(ll.begin(), ll.end(), raw + G + 2 * n);
    }
    if (report) {
        std::memset(report, 0, sizeof *report);
        report->device_status = ctl[2];
        report->elapsed_ms = ms;
    }
    if (ctl[2] & (kStatusTimeoutFlag | kStatusTimeoutDone))
        return set_error(L2D_ERR_PROBE_TIMEOUT, "SM probe wait timed out (status 0x%x)", ctl[2]);
    l2d_sm_probe_report rep{};
    st = l2d_analyze_sm(G, L, smid.data(), t1.data(), ll.data(), map, cap, &rep);
    rep.device_status = ctl[2];
    rep.elapsed_ms = ms;
    if (report) *report = rep;
    return st;
}

// Probes the address-domain model of [base, base + valid_bytes).  base is 2 MiB aligned; lines are
// only placed below base + valid_bytes.  When no page of the region is complete, the mask is fitted
// on a temporary 4 MiB buffer (its pages are appended after the region's pages and get no attr).
int probe_addr_domains_impl(int device, const uint8_t *base, size_t valid_bytes, const int *sm_map, int num_sm,
                            uint32_t *mask, int *attr, size_t cap_pages, size_t *num_pages_out,
                            const l2d_probe_opts *opts, l2d_addr_probe_report *report, uint32_t *raw, size_t raw_cap,
                            size_t *raw_len) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", device);
    if (!base || valid_bytes == 0) return set_error(L2D_ERR_INVALID, "empty region");
    if (reinterpret_cast<uintptr_t>(base) % kPageBytes) return set_error(L2D_ERR_INVALID, "base must be 2 MiB aligned");
    const size_t num_pages = (valid_bytes + kPageBytes - 1) / kPageBytes;
    if (num_pages_out) *num_pages_out = num_pages;
    if (!attr) return L2D_OK;
    if (!mask || cap_pages < num_pages) return set_error(L2D_ERR_INVALID, "attr capacity %zu < %zu pages", cap_pages, num_pages);
    if (!sm_map || num_sm <= 0 || num_sm > kMaxSmid) return set_error(L2D_ERR_INVALID, "bad SM map");
    DeviceGuard guard(device);
    int G = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, device));
    int ndom[2] = {0, 0};
    std::vector<int> dom(kMaxSmid, -1);
    for (int s = 0; s < num_sm; ++s) {
        if (sm_map[s] != 0 && sm_map[s] != 1) return set_error(L2D_ERR_INVALID, "SM map entry %d is not 0/1", s);
        dom[s] = sm_map[s];
        ndom[sm_map[s]]++;
    }
    if (num_sm != G) return set_error(L2D_ERR_INVALID, "SM map has %d entries, device has %d SMs", num_sm, G);
    if (ndom[0] == 0 || ndom[1] == 0) return set_error(L2D_ERR_INVALID, "SM map has an empty domain");

    const int lines_per_page = (opts && opts->lines_per_page) ? static_cast<int>(opts->lines_per_page) : 5;
    const int fit_pages_wanted = (opts && opts->mask_pages) ? static_cast<int>(opts->mask_pages) : 4;
    std::mt19937_64 rng(0xadd7e55ull);
    std::vector<uint64_t> off;
    std::vector<uint8_t> kind;
    std::unordered_set<uint64_t> used;
    uint64_t fit_shift = 0;  // offset of the temporary fit buffer relative to base, if used
    // Every page has one warm-up line that is never probed: its last complete line inside the
    // valid part of the page.  A measurer loads it (untimed) before each timed line of that page
    // so the timed access never pays a TLB walk.
    auto page_hi = [&](uint64_t pbase) -> uint64_t {
        if (fit_shift && pbase >= fit_shift) return pbase + kPageBytes;
        uint64_t hi = std::min<uint64_t>(pbase + kPageBytes, valid_bytes);
        return pbase + ((hi - pbase) / 128) * 128;
    };
    auto warm_of = [&](uint64_t o) {
        uint64_t pbase = o & ~(kPageBytes - 1);
        return page_hi(pbase) - 128;
    };
    auto add = [&](uint64_t o, uint8_t k) {
        uint64_t pbase = o & ~(kPageBytes - 1);
        if (page_hi(pbase) < pbase + 256) return;  // no room for a probe line besides the warm line
        if (o + 128 > page_hi(pbase) - 128) return;
        if (!used.insert(o).second) return;
        off.push_back(o);
        kind.push_back(k);
    };
    // Full pages of the region (candidates for the mask fit).
    std::vector<size_t> full;
    for (size_t p = 0; p < num_pages; ++p)
        if ((p + 1) * kPageBytes <= valid_bytes) full.push_back(p);
    DevBuf fit_buf;
    std::vector<size_t> fit_pages;
    if (!full.empty()) {
        int want = std::min<int>(fit_pages_wanted, static_cast<int>(full.size()));
        for (int i = 0; i < want; ++i) fit_pages.push_back(full[(full.size() - 1) * i / std::max(1, want - 1)]);
        std::sort(fit_pages.begin(), fit_pages.end());
        fit_pages.erase(std::unique(fit_pages.begin(), fit_pages.end()), fit_pages.end());
    }
    if (fit_pages.empty()) {
        // Temporary buffer: must sit above base so offsets stay non-negative in one table.
        L2D_CUDA_TRY(fit_buf.alloc(3 * kPageBytes));
        L2D_CUDA_TRY(cudaMemset(fit_buf.p, 0, 3 * kPageBytes));
        uintptr_t fa = (reinterpret_cast<uintptr_t>(fit_buf.p) + kPageBytes - 1) & ~(uintptr_t)(kPageBytes - 1);
        if (fa < reinterpret_cast<uintptr_t>(base))
            return set_error(L2D_ERR_UNSUPPORTED, "region smaller than one page and below the fit buffer");
        fit_shift = fa - reinterpret_cast<uintptr_t>(base);
        fit_pages.push_back(num_pages);  // virtual page index used only for grouping
    }
    for (size_t fp : fit_pages) {
        uint64_t pb = (fit_shift ? fit_shift : fp * kPageBytes);
        add(pb, 0);
        for (int b = kMaskLowBit; b <= kMaskHighBit; ++b) add(pb + (1ull << b), 0);
        for (int r = 0; r < 64; ++r) add(pb + (rng() % (kPageBytes / 128)) * 128, 1);
    }
    // attr votes: the page base plus random lines inside the valid part of every page.
    for (size_t p = 0; p < num_pages; ++p) {
        uint64_t lo = p * kPageBytes, hi = page_hi(lo);
        if (hi < lo + 256) continue;
        uint64_t nlines = (hi - lo) / 128 - 1;  // excluding the warm line
        add(lo, 2);
        for (int r = 1; r < lines_per_page; ++r) add(lo + (rng() % nlines) * 128, 2);
    }
    const size_t n = off.size();
    if (n < 8) return set_error(L2D_ERR_INVALID, "region too small to probe");
    std::vector<uint64_t> warm(n);
    for (size_t i = 0; i < n; ++i) warm[i] = warm_of(off[i]);

    DevBuf d_off, d_warm, d_dom, d_lat, d_ctl, d_sink;
    L2D_CUDA_TRY(d_off.alloc(n * 8));
    L2D_CUDA_TRY(d_warm.alloc(n * 8));
    L2D_CUDA_TRY(d_dom.alloc(kMaxSmid * sizeof(int)));
    L2D_CUDA_TRY(d_lat.alloc(n * 4));
    L2D_CUDA_TRY(d_ctl.alloc(16));
    L2D_CUDA_TRY(d_sink.alloc(static_cast<size_t>(G) * 8));
    L2D_CUDA_TRY(cudaMemcpy(d_off.p, off.data(), n * 8, cudaMemcpyHostToDevice));
    L2D_CUDA_TRY(cudaMemcpy(d_warm.p, warm.data(), n * 8, cudaMemcpyHostToDevice));
    L2D_CUDA_TRY(cudaMemcpy(d_dom.p, dom.data(), kMaxSmid * sizeof(int), cudaMemcpyHostToDevice));
    L2D_CUDA_TRY(cudaMemset(d_lat.p, 0xff, n * 4));
    L2D_CUDA_TRY(cudaMemset(d_ctl.p, 0, 16));
    int st = flush_l2(device, 0);
    if (st != L2D_OK) return st;

    AddrProbeArgs a;
    a.base = base;
    a.off = d_off.as<uint64_t>();
    a.warm = d_warm.as<uint64_t>();
    a.n = static_cast<uint32_t>(n);
    a.sm_domain = d_dom.as<int>();
    a.n_dom[0] = ndom[0];
    a.n_dom[1] = ndom[1];
    a.lat = d_lat.as<uint32_t>();
    a.ctl = d_ctl.as<uint32_t>();
    a.sink = d_sink.as<uint64_t>();
    a.timeout_ns = timeout_ns_of(opts);
    float ms = 0;
    st = launch_one_per_sm(k_probe_addr_domains, a, G, device, &ms);
    if (st != L2D_OK) return st;
    std::vector<uint32_t> lat(n), ctl(4);
    L2D_CUDA_TRY(cudaMemcpy(lat.data(), d_lat.p, n * 4, cudaMemcpyDeviceToHost));
    L2D_CUDA_TRY(cudaMemcpy(ctl.data(), d_ctl.p, 16, cudaMemcpyDeviceToHost));
    size_t need = 3 * n;
    if (raw_len) *raw_len = need;
    if (raw && raw_cap >= need) {
        for (size_t i = 0; i < n; ++i) {
            raw[i] = static_cast<uint32_t>(off[i]);
            raw[n + i] = lat[i];
            raw[2 * n + i] = kind[i];
        }
    }
    if (report) {
        std::memset(report, 0, sizeof *report);
        report->device_status = ctl[3];
        report->elapsed_ms = ms;
    }
    if (ctl[3] & kStatusTimeoutPrime)
        return set_error(L2D_ERR_PROBE_TIMEOUT, "address probe wait timed out (status 0x%x)", ctl[3]);
    if (ctl[3] & kStatusTicket)
        return set_error(L2D_ERR_PROBE_COVERAGE, "address probe saw more CTAs in a domain than the SM map holds");
    if (ctl[0] != static_cast<uint32_t>(ndom[1]) || ctl[1] != static_cast<uint32_t>(ndom[0]))
        return set_error(L2D_ERR_PROBE_COVERAGE, "address probe saw %u/%u CTAs, map has %d/%d", ctl[1], ctl[0], ndom[0],
                         ndom[1]);
    // Offsets of the temporary fit buffer map to the virtual page index num_pages.
    std::vector<uint64_t> aoff(off);
    if (fit_shift)
        for (size_t i = 0; i < n; ++i)
            if (off[i] >= fit_shift) aoff[i] = num_pages * kPageBytes + (off[i] - fit_shift);
    std::vector<int> attr_all(num_pages + 1, 0);
    l2d_addr_probe_report rep{};
    st = l2d_analyze_addr(n, aoff.data(), lat.data(), kind.data(), num_pages + (fit_shift ? 1 : 0), mask,
                          attr_all.data(), &rep);
    rep.device_status = ctl[3];
    rep.elapsed_ms = ms;
    if (report) *report = rep;
    if (st == L2D_OK || st == L2D_ERR_NOT_LINEAR) std::copy(attr_all.begin(), attr_all.begin() + num_pages, attr);
    return st;
}

}  // namespace l2d

using namespace l2d;

extern "C" {

int l2d_probe_sm_domains(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts) {
    clear_error();
    return probe_sm_domains_impl(device, map, cap, num_sm, opts, nullptr, nullptr, 0, nullptr);
}

int l2d_probe_sm_domains_ex(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts,
                            l2d_sm_probe_report *report, uint32_t *raw, size_t raw_cap, size_t *raw_len) {
    clear_error();
    return probe_sm_domains_impl(device, map, cap, num_sm, opts, report, raw, raw_cap, raw_len);
}

int l2d_probe_addr_domains(int device, const void *base, size_t bytes, const int *sm_map, int num_sm, uint32_t *mask,
                           int *attr, size_t cap_pages, size_t *num_pages, const l2d_probe_opts *opts) {
    clear_error();
    if (bytes % kPageBytes) return set_error(L2D_ERR_INVALID, "bytes must be a multiple of 2 MiB");
    return probe_addr_domains_impl(device, static_cast<const uint8_t *>(base), bytes, sm_map, num_sm, mask, attr,
                                   cap_pages, num_pages, opts, nullptr, nullptr, 0, nullptr);
}

int l2d_probe_addr_domains_ex(int device, const void *base, size_t bytes, const int *sm_map, int num_sm,
                              uint32_t *mask, int *attr, size_t cap_pages, size_t *num_pages,
                              const l2d_probe_opts *opts, l2d_addr_probe_report *report, uint32_t *raw,
                              size_t raw_cap, size_t *raw_len) {
    clear_error();
    if (bytes % kPageBytes) return set_error(L2D_ERR_INVALID, "bytes must be a multiple of 2 MiB");
    return probe_addr_domains_impl(device, static_cast<const uint8_t *>(base), bytes, sm_map, num_sm, mask, attr,
                                   cap_pages, num_pages, opts, report, raw, raw_cap, raw_len);
}

}  // extern "C"
