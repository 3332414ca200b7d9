/*
 * l2d.h -- C ABI of libl2d, the B200-native L2-domain-aware GEMV (y = A.x).
 *
 * All entry points are `extern "C"`, take plain pointers and sizes, return an int status
 * (L2D_OK = 0, negative on error) and never abort the process.  The message of the last
 * failure on the calling thread is available from l2d_last_error().
 *
 * Device work is stream-ordered on the caller's cudaStream_t (passed as void*; NULL = the
 * legacy default stream).  A plan belongs to one device and must not be used concurrently
 * from several threads without external locking.
 *
 * Reference interfaces replaced (LyleLuo/L2Domain; paths relative to that project):
 *   l2d_probe_sm_domains    utility/latopt.cuh:532 get_map_smid2side<T>(T*, size_t&) and the
 *                           standalone tool utility/get_smid2side.cu:114-189
 *   l2d_probe_addr_domains  utility/latopt.cuh:784 get_map_memory_attr<T>(...) and the
 *                           standalone tool utility/get_mask.cu:172-267
 *   l2d_predict_far         utility/latopt.cuh:255-263 predict_map_memory_attr_far
 *   l2d_predict_addr_side   applications/gemv/src/gemv_k1024_persistent_subwarp.cu:105-108
 *   l2d_partition_rows      applications/gemv/src/gemv_k1024_persistent_subwarp.cu:261-273
 *   l2d_plan_create         applications/gemv/src/gemv_k1024_persistent_subwarp.cu:73-103 (build_side_info)
 *   l2d_gemv                applications/gemv/src/gemv_k1024_persistent_subwarp.cu:163-231
 *                           (gemv_partitioned_kernel / gemv_baseline_kernel launches, :301-334)
 *   l2d_l2_flush            utility/latopt.cuh:103-134,190 (GlobalL2Cache::reset)
 *   l2d_fill_*              applications/gemv/src/gemv_k1024_persistent_subwarp.cu:118-139 (init_data)
 *   l2d_write_smid2side_csv / l2d_read_smid2side_csv   utility/get_smid2side.cu:163-177 file format
 *   l2d_write_mask_csv / l2d_read_mask_csv             utility/get_mask.cu:242-252 file format
 *   l2d_pool_alloc / l2d_pool_free / l2d_pool_base     utility/sidedgpu.cu:791-882 (cudaMallocSided,
 *                           cudaFreeSided, cudaGetSidedPoolBase; pool growth :685-745, page
 *                           classification :187-276)
 */
#ifndef L2D_H
#define L2D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define L2D_API __attribute__((visibility("default")))
#else
#define L2D_API
#endif

#define L2D_VERSION 100

/* ---- status codes ---- */
enum {
    L2D_OK = 0,
    L2D_ERR_INVALID = -1,          /* bad argument or unsupported shape */
    L2D_ERR_CUDA = -2,             /* CUDA runtime error */
    L2D_ERR_NO_DEVICE = -3,        /* no usable CUDA device */
    L2D_ERR_PROBE_TIMEOUT = -4,    /* a bounded device-side wait ran out */
    L2D_ERR_PROBE_COVERAGE = -5,   /* the probe did not see exactly one CTA per SM */
    L2D_ERR_PROBE_AMBIGUOUS = -6,  /* latencies do not separate into a near and a far class */
    L2D_ERR_UNSUPPORTED = -7,
    L2D_ERR_IO = -8,               /* file read/write or format error */
    L2D_ERR_NCCL = -9,
    L2D_ERR_NOT_LINEAR = -10,      /* the address hash is not XOR-linear within a 2 MiB page */
    L2D_ERR_STALE = -11            /* a cached domain map belongs to another GPU, SM count or driver */
};

/* ---- element types and execution modes ---- */
enum { L2D_F32 = 0, L2D_F16 = 1, L2D_BF16 = 2 };
enum {
    L2D_MODE_OBLIVIOUS = 0, /* domain-oblivious control: same kernel, pseudo-random granule split */
    L2D_MODE_AWARE = 1,     /* every SM streams only granules homed in its own L2 domain */
    L2D_MODE_SWAPPED = 2,   /* negative control: every SM streams only far-domain granules */
    L2D_MODE_STREAM = 3     /* plain streaming GEMV, no split (whole rows per warp) */
};

L2D_API int l2d_version(void);
L2D_API const char *l2d_last_error(void);
L2D_API const char *l2d_status_string(int status);

/* ---- domain probes ---- */
typedef struct {
    uint32_t timeout_ms;      /* bound of every device-side wait (0 = 1000 ms) */
    uint32_t lines_per_sm;    /* probe lines per SM for the SM map (0 = 48) */
    uint32_t lines_per_page;  /* attr votes per 2 MiB page (0 = 5) */
    uint32_t mask_pages;      /* pages used to fit the mask (0 = 4) */
    uint32_t reserved[4];
} l2d_probe_opts;

enum { L2D_BEHAVIOR_UNKNOWN = 0, L2D_BEHAVIOR_HOME_ONLY = 1, L2D_BEHAVIOR_NEAR_COPY = 2 };

typedef struct {
    int num_sm;              /* SMs seen (one CTA each) */
    int leader_smid;         /* SM that primed the lines */
    int behavior;            /* L2D_BEHAVIOR_*: whether an L2 half keeps copies of far lines */
    int domain_sms[2];       /* SMs per domain (domain 0 = the domain of SM 0) */
    float near_cycles;       /* mean latency of the near class */
    float far_cycles;        /* mean latency of the far class */
    float threshold;         /* 2-means split point */
    float separation;        /* (far - near) / pooled standard deviation */
    float min_agreement;     /* worst per-SM vote agreement in [0, 1] */
    uint32_t device_status;  /* device status bits (timeouts) */
    double elapsed_ms;       /* wall time of the probe kernel */
} l2d_sm_probe_report;

typedef struct {
    uint32_t mask;           /* within-page hash bits */
    int granule_shift;       /* log2 of the smallest domain-uniform block (lowest mask bit, 21 if mask = 0) */
    float near_cycles, far_cycles, threshold, separation;
    float mask_agreement;    /* share of random validation lines the linear model predicts */
    float attr_agreement;    /* worst per-page vote agreement */
    double domain1_fraction; /* share of the region's granules homed in domain 1 */
    uint32_t device_status;
    double elapsed_ms;
} l2d_addr_probe_report;

/* SM -> L2 domain map (replaces latopt.cuh:532).  map[smid] in {0, 1}; domain 0 is SM 0's.
 * `cap` entries are available in map; *num_sm receives the SM count.  map == NULL only queries
 * *num_sm.  report and raw are optional; raw receives, when raw_cap allows, the CTA->smid list
 * followed by the target-first, target-second and leader latency matrices (uint32 cycles). */
L2D_API int l2d_probe_sm_domains(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts);
L2D_API int l2d_probe_sm_domains_ex(int device, int *map, int cap, int *num_sm, const l2d_probe_opts *opts,
                                    l2d_sm_probe_report *report, uint32_t *raw, size_t raw_cap, size_t *raw_len);

/* Address -> L2 domain model of the region [base, base+bytes) (replaces latopt.cuh:784).
 * base must be 2 MiB aligned.  attr receives one entry per 2 MiB page (cap_pages entries);
 * *num_pages receives the page count.  attr == NULL only queries *num_pages. */
L2D_API int l2d_probe_addr_domains(int device, const void *base, size_t bytes, const int *sm_map, int num_sm,
                                   uint32_t *mask, int *attr, size_t cap_pages, size_t *num_pages,
                                   const l2d_probe_opts *opts);
L2D_API int l2d_probe_addr_domains_ex(int device, const void *base, size_t bytes, const int *sm_map, int num_sm,
                                      uint32_t *mask, int *attr, size_t cap_pages, size_t *num_pages,
                                      const l2d_probe_opts *opts, l2d_addr_probe_report *report, uint32_t *raw,
                                      size_t raw_cap, size_t *raw_len);

/* Host-side analysis used by the probes, exported so it can be tested without a GPU.
 * l2d_analyze_sm: lat_* are [n_cta x lines] matrices; smid_of_cta[n_cta]; writes map[smid]. */
L2D_API int l2d_analyze_sm(int n_cta, int lines, const uint32_t *smid_of_cta, const uint32_t *lat_target,
                           const uint32_t *lat_leader, int *map, int map_cap, l2d_sm_probe_report *report);
/* l2d_analyze_addr: offsets[n] (bytes from base), lat[n] measured from domain 0, kind[n]:
 * 0 = mask-fit line of page page_of[n] (offset 0 and 2^b), 1 = validation line, 2 = attr vote. */
L2D_API int l2d_analyze_addr(size_t n, const uint64_t *offsets, const uint32_t *lat, const uint8_t *kind,
                             size_t num_pages, uint32_t *mask, int *attr, l2d_addr_probe_report *report);
/* 2-means split of a latency sample; returns L2D_ERR_PROBE_AMBIGUOUS when the classes overlap. */
L2D_API int l2d_kmeans2(const uint32_t *lat, size_t n, float *threshold, float *near_mean, float *far_mean,
                        float *separation);

/* ---- predictor and placement (host) ---- */
L2D_API int l2d_predict_far(int side, uint32_t mask, uint64_t addr, int attr);
L2D_API int l2d_predict_addr_side(uint64_t base, uint32_t mask, const int *attr, size_t n_attr, uint64_t addr);
L2D_API int l2d_partition_rows(uint64_t base, uint64_t row_bytes, int64_t M, uint32_t mask, const int *attr,
                               size_t n_attr, int32_t *side0, int64_t *n0, int32_t *side1, int64_t *n1,
                               int32_t *base0, int64_t *nb0, int32_t *base1, int64_t *nb1);

/* ---- calibration files in the reference formats ---- */
L2D_API int l2d_write_smid2side_csv(const char *path, const int *map, int num_sm);
L2D_API int l2d_read_smid2side_csv(const char *path, int *map, int cap, int *num_sm);
L2D_API int l2d_write_mask_csv(const char *path, uint32_t mask);
L2D_API int l2d_read_mask_csv(const char *path, uint32_t *mask);

/* ---- domain-map cache (replaces utility/sidedgpu.cu:278-300 read_smid2side, :487-507 read_mask,
 *      :118-130 the $SIDEDGPU_CONFIG_DIR lookup) ----
 * A cache directory holds smid2side.csv and mask.csv in the reference formats plus l2d_device.txt,
 * one line naming the device the map was probed on (l2d_device_key).  The reference trusts any
 * smid2side.csv whose entry count equals the SM count; here a map is reused only when the key
 * matches too, so a map probed on another GPU, after a driver update or under a different SM count
 * is never applied.  When $SIDEDGPU_CONFIG_DIR is set, l2d_plan_create reads the cache instead of
 * running the SM probe (l2d_plan_stats.sm_map_cached) and probes when it is missing, corrupt or
 * stale; the calibration tools write it. */
#define L2D_DEVICE_KEY_MAX 256
/* "uuid=GPU-...;sm=148;cc=10.0;cuda_driver=12090;name=..." for a device. */
L2D_API int l2d_device_key(int device, char *key, int cap);
/* Reads the cache in dir and checks it against key (NULL: skip the identity check, as the reference
 * does) and num_sm (0: skip).  L2D_ERR_IO: a file is missing or malformed; L2D_ERR_STALE: the key or
 * the SM count differs, or a domain has no SM.  mask may be NULL (mask.csv then is not read). */
L2D_API int l2d_domain_cache_check(const char *dir, const char *key, int num_sm, int *map, int cap, int *num_sm_out,
                                   uint32_t *mask);
/* Writes smid2side.csv, mask.csv and l2d_device.txt into dir (which must exist). */
L2D_API int l2d_domain_cache_store(const char *dir, const char *key, const int *map, int num_sm, uint32_t mask);
/* l2d_domain_cache_check against this device's key and SM count. */
L2D_API int l2d_domain_cache_load(int device, const char *dir, int *map, int cap, int *num_sm, uint32_t *mask);

/* ---- GEMV plans ---- */
typedef struct l2d_plan l2d_plan;

typedef struct {
    int64_t M;          /* rows per problem */
    int64_t N;          /* columns (the reference's K) */
    int64_t lda;        /* elements between rows (>= N; 0 = N) */
    int dtype_in;       /* A and x storage: L2D_F32 / L2D_F16 / L2D_BF16 */
    int dtype_out;      /* y storage */
    int64_t batch;      /* independent problems (0 or 1 = single) */
    int64_t stride_a;   /* elements between consecutive problems' A (0 = M*lda) */
    int64_t stride_x;   /* elements between consecutive x (0 = N) */
    int64_t stride_y;   /* elements between consecutive y (0 = M) */
    int device;
    const void *A;      /* the A allocation the plan's domain map describes */
    int flags;          /* L2D_PLAN_* */
} l2d_gemv_desc;

enum {
    L2D_PLAN_NO_PROBE = 1, /* skip the domain probes: only L2D_MODE_STREAM is available */
    L2D_PLAN_TMA = 2,      /* use the granule-ring kernels (A streamed by TMA bulk copies into per-warp
                              shared-memory rings) for every mode when the shape allows them (rows on
                              4 KiB boundaries, x in shared memory); by default the plan picks them
                              per call where they were measured faster */
    L2D_PLAN_NO_TMA = 4,   /* never use the granule-ring kernels */
    /* Placement of the split modes (AWARE, SWAPPED, OBLIVIOUS); by default the plan picks it from
     * A's size against the L2 (see l2d_plan_stats.placement). */
    L2D_PLAN_GRANULES = 8, /* every 4 KiB granule goes to the group of its domain: an SM reads only
                              its own domain's granules, rows that span both domains are summed in
                              two parts */
    L2D_PLAN_ROWS = 16     /* every row goes whole to the group of its first granule's domain (the
                              reference's placement, gemv_k1024_persistent_subwarp.cu:264-269) */
};

typedef struct {
    int num_sm;
    const int *sm_domain;   /* [num_sm] */
    uint32_t mask;
    const int *attr;        /* [num_pages] per 2 MiB page of the region starting at base */
    size_t num_pages;
    const void *base;       /* 2 MiB aligned; must cover every row of A */
} l2d_domain_map;

typedef struct {
    int64_t rows_total;          /* batch * M */
    int granule_shift;
    int64_t domain_bytes[2];     /* A bytes homed in each domain */
    int64_t split_rows;          /* rows with granules in both domains */
    int domain_sms[2];
    int grid, block;
    size_t scratch_bytes;        /* device scratch the plan owns */
    uint64_t fallback_slots;     /* slots processed away from their home SM so far */
    uint64_t calls;              /* completed kernel calls (device epoch) */
    int tma;                     /* granule-ring kernels: 0 unavailable, 1 picked per call, 2 every call */
    uint64_t device_errors;      /* bit 0: a granule-ring wait ran out of time (never expected) */
    int ring_modes;              /* bit m set: calls in mode m run the granule-ring kernels */
    int64_t ring_whole_rows;     /* ring calls in AWARE / OBLIVIOUS: the last rows, taken whole by either group */
    int64_t ring_chunk_rows;     /* ring calls: rows per claim from a row pool */
    int sm_map_cached;           /* 1: the SM map was read from the domain-map cache, 0: probed or given */
    int placement;               /* split modes: 0 granules, 1 whole rows (L2D_PLAN_GRANULES / _ROWS) */
    int64_t row_domain_bytes[2]; /* A bytes in rows whose first granule is homed in each domain */
} l2d_plan_stats;

/* Creates a plan.  map == NULL probes the device and desc->A's region (2 MiB pages covering
 * every row).  The plan owns its device scratch (allocated here, never during l2d_gemv). */
L2D_API int l2d_plan_create(const l2d_gemv_desc *desc, const l2d_domain_map *map, l2d_plan **plan);
L2D_API int l2d_plan_destroy(l2d_plan *plan);
/* y = A.x for every problem, stream-ordered; A must be desc->A (the planned allocation). */
L2D_API int l2d_gemv(l2d_plan *plan, const void *A, const void *x, void *y, int mode, void *stream);
/* Synchronises the device and reads the plan's device counters into *stats. */
L2D_API int l2d_plan_stats_get(l2d_plan *plan, l2d_plan_stats *stats);
/* The plan's SM->domain map and mask/attr (for the CLI and the calibration files). */
L2D_API int l2d_plan_domain_map(const l2d_plan *plan, int *sm_domain, int cap, int *num_sm, uint32_t *mask);

/* ---- allocation-free GEMV (no counterpart in the reference) ----
 * For callers that cannot allocate device memory when they run a GEMV: serving runtimes that
 * reserve all HBM for their own pools at start-up and forbid later allocations, and latency-
 * critical paths that must not enter the allocator (cudaMalloc can synchronise the device).  Same
 * kernel and modes as l2d_gemv, but no plan: the scratch is a file-scope device array of the
 * library (about 1.6 MiB per GPU, held until exit), so the call allocates nothing.  The caller
 * passes A (desc->A), x, y and, for every mode but STREAM, the domain map (l2d_probe_sm_domains /
 * l2d_probe_addr_domains output; map may be NULL for STREAM).  Each call launches a one-CTA
 * set-up kernel that receives the call's SM->slot table and attr bits as kernel parameters, then
 * the GEMV kernel; nothing is copied from host memory.  The first call on a device looks up the
 * array's address (cudaGetSymbolAddress) and clears it, and waits for that to finish; later calls
 * only enqueue work.  Make that first call on each device before any stream capture begins.
 * Calls share the array and each leaves its contents for the next: calls that overlap on the GPU
 * (other streams, other threads) race and must be serialised by the caller.  Sizes beyond the
 * limits below return L2D_ERR_INVALID. */
#define L2D_NOALLOC_MAX_ROWS 196608  /* batch * M */
#define L2D_NOALLOC_MAX_PAGES 32768  /* 2 MiB pages spanned by the domain map (64 GiB of A) */
L2D_API int l2d_gemv_noalloc(const l2d_gemv_desc *desc, const l2d_domain_map *map, const void *x, void *y,
                             int mode, void *stream);

/* ---- sided matrices: the domain-classified placement of utility/sidedgpu.cu:791-838 (cudaMallocSided,
 *      which hands out 4 KiB granules homed in one L2 domain) applied to the GEMV's A ----
 * A dense row-major M x N matrix is packed once (l2d_sided_pack) into a buffer the object owns, where
 * rows [0, rows_side[0]) sit only in granules homed in L2 domain 0 and the other rows only in
 * granules homed in domain 1: contiguous row ranges per domain instead of index lists.  The buffer is
 * as large as A (every granule is used; each side takes one granule of every 8 KiB pair, which the
 * address hash always splits between the domains).  l2d_gemv_sided computes y = A.x from it: AWARE
 * streams each domain's rows on that domain's SMs -- whole rows, near granules only, no per-row
 * partials -- and a group that finishes first takes over the other side's remaining rows; SWAPPED
 * starts every group on the far side (the control); STREAM (and OBLIVIOUS, the same for whole rows)
 * hands rows to any SM.  Every mode computes each row in one warp with its granules in order, so
 * all modes give the same bits, equal to l2d_gemv's STREAM on the dense A (except on the last rows
 * of a large dense call on rows of 8+ granules, which l2d_gemv sums in two halves).  Rows must be
 * whole 4 KiB granules, at most 96 KiB (x is staged in shared memory); one problem. */
typedef struct l2d_sided l2d_sided;
typedef struct {
    int64_t rows_side[2];   /* rows stored in domain-0 and domain-1 granules */
    int granules_per_row;
    const void *base;       /* the packed buffer (2 MiB aligned) */
    size_t bytes;
    uint32_t mask;          /* the address hash the layout follows */
} l2d_sided_info_t;
/* desc: M, N, dtype_in, dtype_out, device (lda, strides, A and flags are ignored; batch <= 1).
 * Allocates the buffer and probes its pages' domains (and the SM map unless it is cached). */
L2D_API int l2d_sided_create(const l2d_gemv_desc *desc, l2d_sided **out);
/* The same with the buffer taken from the device's domain-classified pool (l2d_pool_*, the role of
 * cudaMallocSided, utility/sidedgpu.cu:791-838): a run of whole free 2 MiB pages (the pool grows
 * 1 GiB at a time as needed; opts tunes the probes of new chunks, NULL = defaults), each side's rows
 * then in granules the pool classified as that side -- checked granule by granule at creation
 * (L2D_ERR_PROBE_AMBIGUOUS if the pool and the layout disagree).  l2d_sided_destroy returns the
 * pages to the pool. */
L2D_API int l2d_sided_create_pooled(const l2d_gemv_desc *desc, const l2d_probe_opts *opts, l2d_sided **out);
/* Copies the dense row-major A (lda elements per row, 0 = N) into the sided layout, stream-ordered. */
L2D_API int l2d_sided_pack(l2d_sided *s, const void *A, int64_t lda, void *stream);
L2D_API int l2d_gemv_sided(l2d_sided *s, const void *x, void *y, int mode, void *stream);
L2D_API int l2d_sided_info(const l2d_sided *s, l2d_sided_info_t *info);
/* Device addresses of the granules holding row `row` (granules_per_row entries, in row order). */
L2D_API int l2d_sided_row_granules(const l2d_sided *s, int64_t row, uint64_t *addr, int cap, int *n);
L2D_API int l2d_sided_destroy(l2d_sided *s);

/* ---- row-sharded GEMV over the GPUs of one node (peer memory; no counterpart in the reference) ----
 * One process (or one shard object) per GPU.  Rank r owns rows [row0, row0 + rows) of an M_total-row
 * problem; its plan covers exactly those rows (desc.M = rows, desc.A = its rows of A).  Each rank:
 *   l2d_shard_create -> l2d_shard_handle (exchange the blobs, e.g. an all_gather of bytes)
 *   -> l2d_shard_connect(all blobs in rank order) -> per step:
 *      rank 0 writes x into l2d_shard_buffers(l2d_shard_next_parity()) .x, then every rank calls
 *      l2d_gemv_sharded; after it (stream-ordered) the gathered y of all M_total rows is in that
 *      parity's .y buffer on every rank.  Consume it on the same stream before the next step.
 * One kernel per rank and step: rank 0's CTAs store x into every peer's memory over NVLink, each
 * final y row is stored into every peer's memory as it is finished, and every CTA collects its share
 * of the other ranks' rows at its end; each transfer is a flagged 8-byte word the reader retries
 * until it carries the step, so no fence or counter is involved.  Every retry is bounded by
 * timeout_ms (0 = 2000 ms); a timeout sets a bit in l2d_shard_status (1: x never arrived, 2: a
 * peer's rows never arrived) and the kernel returns, leaving the context usable.  Peers only store
 * into each other's memory; nothing loads from a peer. */
typedef struct l2d_shard l2d_shard;
L2D_API int l2d_shard_create(int device, int rank, int world, int64_t M_total, int64_t row0, int64_t rows,
                             int64_t N, int dtype_in, int dtype_out, uint32_t timeout_ms, l2d_shard **shard);
/* Writes this rank's exchange blob (an IPC handle plus layout) into blob; *len = its size.  With
 * blob == NULL only *len is set. */
L2D_API int l2d_shard_handle(const l2d_shard *shard, void *blob, size_t cap, size_t *len);
/* blobs: world blobs of blob_len bytes, in rank order (this rank's own included). */
L2D_API int l2d_shard_connect(l2d_shard *shard, const void *blobs, size_t blob_len);
/* This rank's x (N elements of dtype_in) and gathered y (M_total of dtype_out) of one parity. */
L2D_API int l2d_shard_buffers(const l2d_shard *shard, int parity, void **x, void **y);
L2D_API int l2d_shard_next_parity(const l2d_shard *shard);
/* One step on the plan's stream order; *parity (may be NULL) receives the buffers' parity used. */
L2D_API int l2d_gemv_sharded(l2d_plan *plan, l2d_shard *shard, int mode, void *stream, int *parity);
/* Synchronizes the device, then reads the timeout bits. */
L2D_API int l2d_shard_status(l2d_shard *shard, uint32_t *status);
L2D_API int l2d_shard_destroy(l2d_shard *shard);

/* ---- domain-classified memory pool (replaces utility/sidedgpu.cu:791-882: cudaMallocSided,
 *      cudaFreeSided, cudaGetSidedPoolBase) ----
 * One pool per device: 64 GiB of virtual addresses, backed 1 GiB at a time (CUDA virtual memory
 * API); each new chunk is classified by l2d_probe_addr_domains and every 4 KiB granule gets its L2
 * domain (side).  l2d_pool_alloc hands out ceil(bytes / 4096) free granules of one side as indices
 * from the pool base (granule g lives at base + g * 4096); cap must hold that many.  Not
 * thread-safe across processes; thread-safe within one.  Unlike the reference, errors come back as
 * status codes and a hash finer than 4 KiB is refused (L2D_ERR_UNSUPPORTED). */
L2D_API int l2d_pool_alloc(int device, size_t bytes, int side, const l2d_probe_opts *opts, uint64_t *granules,
                           size_t cap, size_t *count);
L2D_API int l2d_pool_free(int device, const uint64_t *granules, size_t count);
L2D_API int l2d_pool_base(int device, void **base);
/* Mapped bytes, free granules per side ([2]) and the pool's mask; any pointer may be NULL. */
L2D_API int l2d_pool_info(int device, uint64_t *mapped_bytes, uint64_t *free_granules, uint32_t *mask);
/* The side the pool classified each granule as. */
L2D_API int l2d_pool_side(int device, const uint64_t *granules, size_t count, int *sides);
/* Unmaps and frees the whole pool (every granule must be free). */
L2D_API int l2d_pool_release(int device);

/* ---- helpers used by the benchmark and the CLI ---- */
/* Reference-mode inputs (init_data): A/x from mix32 of the flat index (stream 0 = A, 1 = x). */
L2D_API int l2d_fill_ref(void *dst, int dtype, uint64_t first, uint64_t n, uint32_t seed, int stream,
                         int integer_mode, void *stream_handle);
/* BASELINE-config inputs: dist 0 uniform[p0,p1], 1 normal(mean p0, sigma p1), rounded to dtype. */
L2D_API int l2d_fill_cfg(void *dst, int dtype, uint64_t first, uint64_t n, uint64_t seed, uint64_t rng_stream,
                         int dist, float p0, float p1, void *stream_handle);
/* Evicts the L2 by writing a device buffer of the L2's size (GlobalL2Cache::reset). */
L2D_API int l2d_l2_flush(int device, void *stream_handle);
/* Read-only stream over [p, p + bytes), `passes` times in one launch: every byte is read by 32-byte
 * loads, one XOR word per CTA lands in sink (one CTA per SM: sink_words >= the SM count).  p 32-byte
 * aligned, bytes a multiple of 32.  The bandwidth denominator of a read-dominated kernel: HBM read
 * bandwidth over a buffer larger than L2 (passes = 1), L2 read bandwidth over an L2-resident
 * buffer read many times in one launch. */
L2D_API int l2d_read_stream(int device, const void *p, size_t bytes, int passes, uint32_t *sink, size_t sink_words,
                            void *stream_handle);
/* Device properties the roofline needs. */
L2D_API int l2d_device_info(int device, int *num_sm, int *l2_bytes, int *cc_major, int *cc_minor, char *name,
                            int name_cap);

#ifdef __cplusplus
}
#endif
#endif /* L2D_H */
