// Input generators, the L2 flush and device information.
//
// l2d_fill_ref restates init_data (applications/gemv/src/gemv_k1024_persistent_subwarp.cu:118-139):
// A[i] = (mix32(uint32(i) ^ seed) & 0xff) / 255 - 0.5 (x uses seed + 0x9e37), or the exact-integer
// mode of :122-134.  l2d_fill_cfg draws the BASELINE distributions from a counter-based
// splitmix64 stream; the normal draw is Box-Muller with a textbook log series and a Taylor cosine,
// every operation written with explicit round-to-nearest intrinsics so the host generator
// computes identical values.  Storage rounding is IEEE round-to-nearest-even.
#include "l2d_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>

namespace l2d {
namespace gen {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double dfma_free(double p, double s2, double c) { return __dadd_rn(__dmul_rn(p, s2), c); }

__device__ double log_pos(double u) {
    uint64_t bits = static_cast<uint64_t>(__double_as_longlong(u));
    int e = static_cast<int>((bits >> 52) & 0x7ff) - 1023;
    uint64_t mbits = (bits & 0x000fffffffffffffull) | 0x3ff0000000000000ull;
    double m = __longlong_as_double(static_cast<long long>(mbits));
    if (m > 1.4142135623730951) {
        m = __dmul_rn(m, 0.5);
        e = e + 1;
    }
    double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    double s2 = __dmul_rn(s, s);
    double p = 1.0 / 23.0;
    p = dfma_free(p, s2, 1.0 / 21.0);
    p = dfma_free(p, s2, 1.0 / 19.0);
    p = dfma_free(p, s2, 1.0 / 17.0);
    p = dfma_free(p, s2, 1.0 / 15.0);
    p = dfma_free(p, s2, 1.0 / 13.0);
    p = dfma_free(p, s2, 1.0 / 11.0);
    p = dfma_free(p, s2, 1.0 / 9.0);
    p = dfma_free(p, s2, 1.0 / 7.0);
    p = dfma_free(p, s2, 1.0 / 5.0);
    p = dfma_free(p, s2, 1.0 / 3.0);
    p = dfma_free(p, s2, 1.0);
    double lm = __dmul_rn(__dmul_rn(2.0, s), p);
    return __dadd_rn(__dmul_rn(static_cast<double>(e), 0.6931471805599453), lm);
}

// sum_k (-1)^k x^(2k) / (2k)!, k = 0..9, Horner in x^2.
__device__ double cos_series(double x) {
    double x2 = __dmul_rn(x, x);
    double p = -1.0 / 6402373705728000.0;
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 20922789888000.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 87178291200.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 479001600.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 3628800.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 40320.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 720.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 24.0);
    p = __dsub_rn(__dmul_rn(p, x2), 0.5);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0);
    return p;
}

// x * sum_k (-1)^k x^(2k) / (2k+1)!, k = 0..9.
__device__ double sin_series(double x) {
    double x2 = __dmul_rn(x, x);
    double p = -1.0 / 121645100408832000.0;
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 355687428096000.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 1307674368000.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 6227020800.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 39916800.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 362880.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 5040.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0 / 120.0);
    p = __dsub_rn(__dmul_rn(p, x2), 1.0 / 6.0);
    p = __dadd_rn(__dmul_rn(p, x2), 1.0);
    return __dmul_rn(p, x);
}

__device__ double cos_2pi(double u) {
    double w = __dsub_rn(u, 0.5);
    double sign = -1.0;
    if (w < 0.0) w = -w;
    if (w > 0.25) {
        w = __dsub_rn(0.5, w);
        sign = -sign;
    }
    if (w > 0.125) return __dmul_rn(sign, sin_series(__dmul_rn(__dsub_rn(0.25, w), 6.283185307179586)));
    return __dmul_rn(sign, cos_series(__dmul_rn(w, 6.283185307179586)));
}

__device__ __forceinline__ uint64_t rng_u64(uint64_t seed, uint64_t stream, uint64_t index, uint32_t sub) {
    uint64_t key = splitmix64(seed ^ (stream * 0xd1342543de82ef95ull) ^ 0x243f6a8885a308d3ull);
    return splitmix64(key + 2ull * index + sub);
}

__device__ float cfg_value(uint64_t seed, uint64_t stream, uint64_t index, int dist, float p0, float p1) {
    uint64_t r0 = rng_u64(seed, stream, index, 0);
    if (dist == 0) {
        float u = __fmul_rn(__uint2float_rn(static_cast<uint32_t>(r0 >> 40)), 0x1p-24f);
        float span = __fsub_rn(p1, p0);
        return __fadd_rn(p0, __fmul_rn(span, u));
    }
    uint64_t r1 = rng_u64(seed, stream, index, 1);
    double u1 = __dmul_rn(__ull2double_rn((r0 >> 11) + 1ull), 0x1p-53);
    double u2 = __dmul_rn(__ull2double_rn(r1 >> 11), 0x1p-53);
    double l = log_pos(u1);
    double r = __dsqrt_rn(__dmul_rn(-2.0, l));
    double z = __dmul_rn(r, cos_2pi(u2));
    double v = __dadd_rn(__dmul_rn(static_cast<double>(p1), z), static_cast<double>(p0));
    return __double2float_rn(v);
}

__device__ __forceinline__ void store(void *dst, int dtype, uint64_t j, float v) {
    if (dtype == L2D_F32) static_cast<float *>(dst)[j] = v;
    else if (dtype == L2D_F16) static_cast<__half *>(dst)[j] = __float2half_rn(v);
    else static_cast<__nv_bfloat16 *>(dst)[j] = __float2bfloat16_rn(v);
}

__global__ void k_fill_ref(void *dst, int dtype, uint64_t first, uint64_t n, uint32_t seed, int stream, int integer) {
    const uint32_t s = stream == 0 ? seed : seed + 0x9e37u;
    for (uint64_t j = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; j < n;
         j += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        uint32_t h = mix32(static_cast<uint32_t>(first + j) ^ s);
        float v;
        if (integer) v = stream == 0 ? static_cast<float>(static_cast<int>(h % 17u) - 8)
                                     : static_cast<float>(static_cast<int>(h % 7u) - 3);
        else v = __fsub_rn(__fdiv_rn(__uint2float_rn(h & 0xffu), 255.0f), 0.5f);
        store(dst, dtype, j, v);
    }
}

__global__ void k_fill_cfg(void *dst, int dtype, uint64_t first, uint64_t n, uint64_t seed, uint64_t rs, int dist,
                           float p0, float p1) {
    for (uint64_t j = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; j < n;
         j += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        store(dst, dtype, j, cfg_value(seed, rs, first + j, dist, p0, p1));
}

int fill_grid(uint64_t n) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    uint64_t want = (n + 255) / 256;
    uint64_t cap = static_cast<uint64_t>(sms) * 16;
    return static_cast<int>(want < cap ? (want ? want : 1) : cap);
}

std::mutex g_flush_mu;
std::map<int, std::pair<void *, size_t>> g_flush;  // device -> flush buffer (kept until exit)

// Read-only stream: every 32-byte chunk of [p, p + n32 * 32) is loaded once per pass (256-bit
// non-coherent loads that do not allocate in L1, 4 in flight per thread, 128 KiB per SM) and folded
// into one XOR word per CTA, so the loads cannot be elided.  The roofline denominators for a
// read-dominated kernel: over a buffer larger than L2 it gives the HBM read bandwidth; over an
// L2-resident buffer read `passes` times in one launch, the L2 read bandwidth without the launch in
// it (no load allocates in L1, so a repeated pass is served by L2, not by the SM's own cache).
__device__ __forceinline__ uint32_t ld_xor32(const uint8_t *q) {
    uint32_t v[8];
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "l"(q));
    return v[0] ^ v[1] ^ v[2] ^ v[3] ^ v[4] ^ v[5] ^ v[6] ^ v[7];
}

__global__ void __launch_bounds__(1024) k_read_stream(const uint8_t *p, uint64_t n32, uint32_t *sink, int passes) {
    constexpr int kU = 4;
    uint32_t acc = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (int pass = 0; pass < passes; ++pass) {
        uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
        for (; i + (kU - 1) * stride < n32; i += kU * stride) {
            uint32_t v[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) v[u] = ld_xor32(p + (i + u * stride) * 32);
#pragma unroll
            for (int u = 0; u < kU; ++u) acc ^= v[u];
        }
        for (; i < n32; i += stride) acc ^= ld_xor32(p + i * 32);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ uint32_t s[32];
    if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t ^= s[w];
        sink[blockIdx.x] = t;
    }
}

}  // namespace gen
}  // namespace l2d

using namespace l2d;

extern "C" {

int l2d_fill_ref(void *dst, int dtype, uint64_t first, uint64_t n, uint32_t seed, int stream, int integer_mode,
                 void *stream_handle) {
    clear_error();
    if (!valid_dtype(dtype)) return set_error(L2D_ERR_INVALID, "bad dtype");
    if (n == 0) return L2D_OK;
    if (!dst) return set_error(L2D_ERR_INVALID, "null destination");
    gen::k_fill_ref<<<gen::fill_grid(n), 256, 0, static_cast<cudaStream_t>(stream_handle)>>>(dst, dtype, first, n,
                                                                                           seed, stream, integer_mode);
    L2D_CUDA_TRY(cudaGetLastError());
    return L2D_OK;
}

int l2d_fill_cfg(void *dst, int dtype, uint64_t first, uint64_t n, uint64_t seed, uint64_t rng_stream, int dist,
                 float p0, float p1, void *stream_handle) {
    clear_error();
    if (!valid_dtype(dtype) || (dist != 0 && dist != 1)) return set_error(L2D_ERR_INVALID, "bad dtype or dist");
    if (n == 0) return L2D_OK;
    if (!dst) return set_error(L2D_ERR_INVALID, "null destination");
    gen::k_fill_cfg<<<gen::fill_grid(n), 256, 0, static_cast<cudaStream_t>(stream_handle)>>>(dst, dtype, first, n,
                                                                                           seed, rng_stream, dist, p0, p1);
    L2D_CUDA_TRY(cudaGetLastError());
    return L2D_OK;
}

int l2d_l2_flush(int device, void *stream_handle) {
    clear_error();
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) L2D_CUDA_TRY(cudaSetDevice(device));
    std::pair<void *, size_t> buf{nullptr, 0};
    {
        std::lock_guard<std::mutex> lk(gen::g_flush_mu);
        auto it = gen::g_flush.find(device);
        if (it == gen::g_flush.end()) {
            int l2 = 0;
            L2D_CUDA_TRY(cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, device));
            size_t bytes = static_cast<size_t>(l2) * 2;  // both L2 halves, with margin
            void *p = nullptr;
            L2D_CUDA_TRY(cudaMalloc(&p, bytes));
            it = gen::g_flush.emplace(device, std::make_pair(p, bytes)).first;
        }
        buf = it->second;
    }
    cudaError_t e = cudaMemsetAsync(buf.first, 0, buf.second, static_cast<cudaStream_t>(stream_handle));
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "l2_flush: %s", cudaGetErrorString(e));
    return L2D_OK;
}

int l2d_read_stream(int device, const void *p, size_t bytes, int passes, uint32_t *sink, size_t sink_words,
                    void *stream_handle) {
    clear_error();
    if (passes < 1) return set_error(L2D_ERR_INVALID, "read_stream: passes must be >= 1");
    if (!p || !sink || (reinterpret_cast<uintptr_t>(p) & 31) || (bytes & 31))
        return set_error(L2D_ERR_INVALID, "read_stream: p must be 32-byte aligned and bytes a multiple of 32");
    int num_sm = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&num_sm, cudaDevAttrMultiProcessorCount, device));
    if (sink_words < static_cast<size_t>(num_sm))
        return set_error(L2D_ERR_INVALID, "read_stream: sink holds %zu words, needs %d", sink_words, num_sm);
    if (bytes == 0) return L2D_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) L2D_CUDA_TRY(cudaSetDevice(device));
    gen::k_read_stream<<<num_sm, 1024, 0, static_cast<cudaStream_t>(stream_handle)>>>(
        static_cast<const uint8_t *>(p), bytes / 32, sink, passes);
    cudaError_t e = cudaGetLastError();
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(L2D_ERR_CUDA, "read_stream: %s", cudaGetErrorString(e));
    return L2D_OK;
}

int l2d_device_key(int device, char *key, int cap) {
    clear_error();
    if (!key || cap <= 0) return set_error(L2D_ERR_INVALID, "device_key: bad arguments");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", device);
    cudaDeviceProp prop;
    L2D_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    int drv = 0;
    L2D_CUDA_TRY(cudaDriverGetVersion(&drv));
    const unsigned char *u = reinterpret_cast<const unsigned char *>(prop.uuid.bytes);
    char uuid[48];
    std::snprintf(uuid, sizeof uuid, "GPU-%02x%02x%02x%02x-%02x%02x-%02x%02x-%02x%02x-%02x%02x%02x%02x%02x%02x", u[0], u[1],
                  u[2], u[3], u[4], u[5], u[6], u[7], u[8], u[9], u[10], u[11], u[12], u[13], u[14], u[15]);
    const int n = std::snprintf(key, static_cast<size_t>(cap), "uuid=%s;sm=%d;cc=%d.%d;cuda_driver=%d;name=%s", uuid,
                                prop.multiProcessorCount, prop.major, prop.minor, drv, prop.name);
    if (n < 0 || n >= cap) return set_error(L2D_ERR_INVALID, "device_key: capacity %d too small", cap);
    return L2D_OK;
}

int l2d_domain_cache_load(int device, const char *dir, int *map, int cap, int *num_sm, uint32_t *mask) {
    char key[L2D_DEVICE_KEY_MAX + 1];
    int st = l2d_device_key(device, key, sizeof key);
    if (st != L2D_OK) return st;
    int n = 0;
    L2D_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    return l2d_domain_cache_check(dir, key, n, map, cap, num_sm, mask);
}

int l2d_device_info(int device, int *num_sm, int *l2_bytes, int *cc_major, int *cc_minor, char *name, int name_cap) {
    clear_error();
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_error(L2D_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return set_error(L2D_ERR_INVALID, "device %d out of range", device);
    cudaDeviceProp prop;
    L2D_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (num_sm) *num_sm = prop.multiProcessorCount;
    if (l2_bytes) *l2_bytes = prop.l2CacheSize;
    if (cc_major) *cc_major = prop.major;
    if (cc_minor) *cc_minor = prop.minor;
    if (name && name_cap > 0) {
        std::strncpy(name, prop.name, static_cast<size_t>(name_cap) - 1);
        name[name_cap - 1] = '\0';
    }
    return L2D_OK;
}

}  // extern "C"
