// libl2d host core: errors, the domain predictor, row placement, calibration files and the
// latency analysis behind the domain probes.  Pure C++; nothing here touches a GPU, so every
// function is testable on a CPU-only machine through the C ABI.
#include "l2d_internal.h"

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace l2d {

static thread_local std::string g_last_error;

int set_error(int status, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

void clear_error() { g_last_error.clear(); }

}  // namespace l2d

using namespace l2d;

extern "C" {

int l2d_version(void) { return L2D_VERSION; }

const char *l2d_last_error(void) { return g_last_error.c_str(); }

const char *l2d_status_string(int status) {
    switch (status) {
    case L2D_OK: return "ok";
    case L2D_ERR_INVALID: return "invalid argument";
    case L2D_ERR_CUDA: return "CUDA error";
    case L2D_ERR_NO_DEVICE: return "no CUDA device";
    case L2D_ERR_PROBE_TIMEOUT: return "probe wait timed out";
    case L2D_ERR_PROBE_COVERAGE: return "probe did not see one CTA per SM";
    case L2D_ERR_PROBE_AMBIGUOUS: return "latencies do not separate into near and far";
    case L2D_ERR_UNSUPPORTED: return "unsupported";
    case L2D_ERR_IO: return "I/O or format error";
    case L2D_ERR_NCCL: return "NCCL error";
    case L2D_ERR_NOT_LINEAR: return "address hash is not XOR-linear within a page";
    case L2D_ERR_STALE: return "cached domain map belongs to another device or driver";
    default: return "unknown status";
    }
}

// ---------------------------------------------------------------------------------------------
// Predictor and placement (latopt.cuh:255-263; gemv_k1024_persistent_subwarp.cu:105-108, 261-273)
// ---------------------------------------------------------------------------------------------

int l2d_predict_far(int side, uint32_t mask, uint64_t addr, int attr) {
    int parity = __builtin_popcount(static_cast<uint32_t>(addr) & mask) & 1;
    return parity ^ side ^ attr;
}

int l2d_predict_addr_side(uint64_t base, uint32_t mask, const int *attr, size_t n_attr, uint64_t addr) {
    if (!attr || addr < base) return set_error(L2D_ERR_INVALID, "predict_addr_side: address below base");
    uint64_t page = (addr - base) / kPageBytes;
    if (page >= n_attr) return set_error(L2D_ERR_INVALID, "predict_addr_side: page %llu outside the attr table",
                                         (unsigned long long)page);
    return l2d_predict_far(0, mask, addr, attr[page]) & 1;
}

int l2d_partition_rows(uint64_t base, uint64_t row_bytes, int64_t M, uint32_t mask, const int *attr, size_t n_attr,
                       int32_t *side0, int64_t *n0, int32_t *side1, int64_t *n1, int32_t *base0, int64_t *nb0,
                       int32_t *base1, int64_t *nb1) {
    if (M < 0 || !attr || !side0 || !side1 || !base0 || !base1 || !n0 || !n1 || !nb0 || !nb1)
        return set_error(L2D_ERR_INVALID, "partition_rows: null output or negative M");
    if (M > 0 && (M - 1) * row_bytes / kPageBytes >= n_attr)
        return set_error(L2D_ERR_INVALID, "partition_rows: rows extend past the attr table");
    int64_t c0 = 0, c1 = 0, b0 = 0, b1 = 0;
    for (int64_t row = 0; row < M; ++row) {
        uint64_t addr = base + static_cast<uint64_t>(row) * row_bytes;
        int side = l2d_predict_far(0, mask, addr, attr[(addr - base) / kPageBytes]) & 1;
        if (side) side1[c1++] = static_cast<int32_t>(row);
        else side0[c0++] = static_cast<int32_t>(row);
        if (row & 1) base1[b1++] = static_cast<int32_t>(row);
        else base0[b0++] = static_cast<int32_t>(row);
    }
    *n0 = c0;
    *n1 = c1;
    *nb0 = b0;
    *nb1 = b1;
    return L2D_OK;
}

// ---------------------------------------------------------------------------------------------
// Calibration files: smid2side.csv is "%d," per SM then a newline (get_smid2side.cu:170-173);
// mask.csv is "0x%08x\n" (get_mask.cu:248).
// ---------------------------------------------------------------------------------------------

int l2d_write_smid2side_csv(const char *path, const int *map, int num_sm) {
    if (!path || !map || num_sm <= 0) return set_error(L2D_ERR_INVALID, "write_smid2side_csv: bad arguments");
    FILE *f = std::fopen(path, "w");
    if (!f) return set_error(L2D_ERR_IO, "cannot open '%s': %s", path, std::strerror(errno));
    for (int i = 0; i < num_sm; ++i) std::fprintf(f, "%d,", map[i]);
    std::fprintf(f, "\n");
    if (std::fclose(f) != 0) return set_error(L2D_ERR_IO, "cannot close '%s'", path);
    return L2D_OK;
}

int l2d_read_smid2side_csv(const char *path, int *map, int cap, int *num_sm) {
    if (!path || !num_sm) return set_error(L2D_ERR_INVALID, "read_smid2side_csv: bad arguments");
    FILE *f = std::fopen(path, "r");
    if (!f) return set_error(L2D_ERR_IO, "cannot open '%s': %s", path, std::strerror(errno));
    std::vector<int> values;
    int ch;
    std::string tok;
    bool bad = false;
    auto flush_tok = [&]() {
        if (tok.empty()) return;
        char *end = nullptr;
        long v = std::strtol(tok.c_str(), &end, 10);
        if (*end != '\0' || (v != 0 && v != 1)) bad = true;
        else values.push_back(static_cast<int>(v));
        tok.clear();
    };
    while ((ch = std::fgetc(f)) != EOF) {
        if (ch == ',' || ch == '\n' || ch == '\r' || ch == ' ' || ch == '\t') flush_tok();
        else tok.push_back(static_cast<char>(ch));
    }
    flush_tok();
    std::fclose(f);
    if (bad) return set_error(L2D_ERR_IO, "'%s': entries must be 0 or 1", path);
    if (values.empty()) return set_error(L2D_ERR_IO, "'%s': no entries", path);
    *num_sm = static_cast<int>(values.size());
    if (map) {
        if (cap < static_cast<int>(values.size()))
            return set_error(L2D_ERR_INVALID, "'%s' has %zu entries, capacity %d", path, values.size(), cap);
        std::copy(values.begin(), values.end(), map);
    }
    return L2D_OK;
}

int l2d_write_mask_csv(const char *path, uint32_t mask) {
    if (!path) return set_error(L2D_ERR_INVALID, "write_mask_csv: null path");
    FILE *f = std::fopen(path, "w");
    if (!f) return set_error(L2D_ERR_IO, "cannot open '%s': %s", path, std::strerror(errno));
    std::fprintf(f, "0x%08x\n", mask);
    if (std::fclose(f) != 0) return set_error(L2D_ERR_IO, "cannot close '%s'", path);
    return L2D_OK;
}

int l2d_read_mask_csv(const char *path, uint32_t *mask) {
    if (!path || !mask) return set_error(L2D_ERR_INVALID, "read_mask_csv: bad arguments");
    FILE *f = std::fopen(path, "r");
    if (!f) return set_error(L2D_ERR_IO, "cannot open '%s': %s", path, std::strerror(errno));
    char buf[64] = {0};
    size_t n = std::fread(buf, 1, sizeof buf - 1, f);
    std::fclose(f);
    buf[n] = '\0';
    char *p = buf;
    while (*p == ' ' || *p == '\t') ++p;
    if (!(p[0] == '0' && (p[1] == 'x' || p[1] == 'X'))) return set_error(L2D_ERR_IO, "'%s': expected 0x%%08x", path);
    char *end = nullptr;
    errno = 0;
    unsigned long v = std::strtoul(p + 2, &end, 16);
    if (end == p + 2 || errno != 0 || v > 0xffffffffUL) return set_error(L2D_ERR_IO, "'%s': bad mask", path);
    while (*end == '\n' || *end == '\r' || *end == ' ' || *end == '\t') ++end;
    if (*end != '\0') return set_error(L2D_ERR_IO, "'%s': trailing data after the mask", path);
    *mask = static_cast<uint32_t>(v);
    return L2D_OK;
}

// ---------------------------------------------------------------------------------------------
// Latency analysis.  The reference classifies with fixed H100 constants (a 100-cycle spread,
// latopt.cuh:528; above-the-mean, :742-746).  Here every decision uses a 2-means split of the
// measured sample plus a separation test, so the same code serves any near/far gap.
// ---------------------------------------------------------------------------------------------

int l2d_kmeans2(const uint32_t *lat, size_t n, float *threshold, float *near_mean, float *far_mean,
                float *separation) {
    if (!lat || n < 4) return set_error(L2D_ERR_INVALID, "kmeans2: need at least 4 samples");
    std::vector<double> v(lat, lat + n);
    std::sort(v.begin(), v.end());
    // Drop extreme outliers (TLB walks, preemption): anything above 4x the 5th percentile.
    double lo = v[n / 20];
    double cut = 4.0 * std::max(lo, 1.0);
    size_t m = std::upper_bound(v.begin(), v.end(), cut) - v.begin();
    if (m < 4) return set_error(L2D_ERR_PROBE_AMBIGUOUS, "kmeans2: too few samples after outlier removal");
    std::vector<double> pre(m + 1, 0.0), pre2(m + 1, 0.0);
    for (size_t i = 0; i < m; ++i) {
        pre[i + 1] = pre[i] + v[i];
        pre2[i + 1] = pre2[i] + v[i] * v[i];
    }
    double best = INFINITY;
    size_t split = 0;
    for (size_t i = 1; i < m; ++i) {
        double nl = static_cast<double>(i), nr = static_cast<double>(m - i);
        double sl = pre[i], sr = pre[m] - pre[i];
        double ssel = pre2[i] - sl * sl / nl;
        double sser = (pre2[m] - pre2[i]) - sr * sr / nr;
        if (ssel + sser < best) {
            best = ssel + sser;
            split = i;
        }
    }
    double nl = static_cast<double>(split), nr = static_cast<double>(m - split);
    double ml = pre[split] / nl, mr = (pre[m] - pre[split]) / nr;
    double vl = std::max(0.0, pre2[split] / nl - ml * ml), vr = std::max(0.0, (pre2[m] - pre2[split]) / nr - mr * mr);
    double sd = std::sqrt(0.5 * (vl + vr));
    double sep = (mr - ml) / std::max(sd, 1.0);
    if (threshold) *threshold = static_cast<float>(0.5 * (ml + mr));
    if (near_mean) *near_mean = static_cast<float>(ml);
    if (far_mean) *far_mean = static_cast<float>(mr);
    if (separation) *separation = static_cast<float>(sep);
    double minor = std::min(nl, nr) / static_cast<double>(m);
    if (sep < 3.0 || mr - ml < 12.0 || minor < 0.02)
        return set_error(L2D_ERR_PROBE_AMBIGUOUS,
                         "near %.1f / far %.1f cycles, separation %.2f, minor class %.3f: no clear domain split", ml, mr,
                         sep, minor);
    return L2D_OK;
}

int l2d_analyze_sm(int n_cta, int lines, const uint32_t *smid_of_cta, const uint32_t *lat_target,
                   const uint32_t *lat_leader, int *map, int map_cap, l2d_sm_probe_report *report) {
    if (n_cta < 2 || lines < 4 || !smid_of_cta || !lat_target || !lat_leader || !map)
        return set_error(L2D_ERR_INVALID, "analyze_sm: bad arguments");
    // Coverage: one CTA per SM, every smid distinct and inside the map.
    std::vector<int> seen(kMaxSmid, 0);
    for (int c = 0; c < n_cta; ++c) {
        uint32_t s = smid_of_cta[c];
        if (s >= static_cast<uint32_t>(kMaxSmid) || static_cast<int>(s) >= map_cap)
            return set_error(L2D_ERR_PROBE_COVERAGE, "CTA %d reported smid %u outside the map (%d)", c, s, map_cap);
        if (seen[s]++) return set_error(L2D_ERR_PROBE_COVERAGE, "two probe CTAs ran on SM %u", s);
    }
    const size_t per = static_cast<size_t>(lines);
    const size_t total = static_cast<size_t>(n_cta - 1) * per;
    std::vector<uint32_t> pool;
    pool.reserve(2 * total);
    pool.insert(pool.end(), lat_target + per, lat_target + per + total);
    pool.insert(pool.end(), lat_leader + per, lat_leader + per + total);
    float thr = 0, nm = 0, fm = 0, sep = 0;
    int st = l2d_kmeans2(pool.data(), pool.size(), &thr, &nm, &fm, &sep);
    if (report) {
        report->threshold = thr;
        report->near_cycles = nm;
        report->far_cycles = fm;
        report->separation = sep;
        report->leader_smid = static_cast<int>(smid_of_cta[0]);
        report->num_sm = n_cta;
    }
    if (st != L2D_OK) return st;
    size_t lfar = 0;
    for (size_t i = per; i < per + total; ++i) lfar += lat_leader[i] > thr;
    double f_leader = static_cast<double>(lfar) / static_cast<double>(total);
    int behavior = f_leader < 0.05 ? L2D_BEHAVIOR_NEAR_COPY
                   : (f_leader > 0.2 && f_leader < 0.8) ? L2D_BEHAVIOR_HOME_ONLY
                                                        : L2D_BEHAVIOR_UNKNOWN;
    if (report) report->behavior = behavior;
    if (behavior == L2D_BEHAVIOR_UNKNOWN)
        return set_error(L2D_ERR_PROBE_AMBIGUOUS, "leader sees %.3f of its primed lines as far: cannot tell the "
                                                  "cache behaviour", f_leader);
    std::vector<int> rel(n_cta, 0);
    double min_agree = 1.0;
    for (int c = 1; c < n_cta; ++c) {
        const uint32_t *t = lat_target + static_cast<size_t>(c) * per;
        const uint32_t *l = lat_leader + static_cast<size_t>(c) * per;
        double votes = 0;
        if (behavior == L2D_BEHAVIOR_HOME_ONLY) {
            // A line homed in domain h is far for an SM iff h differs from the SM's domain, so
            // far(target) xor far(leader) = domain(target) xor domain(leader) for every line.
            for (size_t j = 0; j < per; ++j) votes += ((t[j] > thr) != (l[j] > thr));
            double f = votes / static_cast<double>(per);
            rel[c] = f > 0.5;
            min_agree = std::min(min_agree, std::max(f, 1.0 - f));
        } else {
            // The leader's half keeps a copy of every line it primed: SMs in the leader's domain
            // see only near hits, the others see the lines homed on the leader's side as far.
            for (size_t j = 0; j < per; ++j) votes += t[j] > thr;
            double f = votes / static_cast<double>(per);
            rel[c] = f > 0.2;
            min_agree = std::min(min_agree, rel[c] ? std::min(1.0, f / 0.3) : 1.0 - f);
        }
    }
    // Re-base so that SM 0 is domain 0, as the reference's map[0] = 0 (latopt.cuh:513).
    int flip = 0;
    for (int c = 0; c < n_cta; ++c)
        if (smid_of_cta[c] == 0) flip = rel[c];
    for (int i = 0; i < map_cap; ++i) map[i] = 0;
    int counts[2] = {0, 0};
    for (int c = 0; c < n_cta; ++c) {
        int d = rel[c] ^ flip;
        map[smid_of_cta[c]] = d;
        counts[d]++;
    }
    if (report) {
        report->domain_sms[0] = counts[0];
        report->domain_sms[1] = counts[1];
        report->min_agreement = static_cast<float>(min_agree);
    }
    if (counts[0] == 0 || counts[1] == 0)
        return set_error(L2D_ERR_PROBE_AMBIGUOUS, "all SMs classified into one domain");
    if (min_agree < 0.8)
        return set_error(L2D_ERR_PROBE_AMBIGUOUS, "an SM's votes agree only %.2f", min_agree);
    return L2D_OK;
}

int l2d_analyze_addr(size_t n, const uint64_t *offsets, const uint32_t *lat, const uint8_t *kind, size_t num_pages,
                     uint32_t *mask_out, int *attr, l2d_addr_probe_report *report) {
    if (n < 8 || !offsets || !lat || !kind || !mask_out || !attr || num_pages == 0)
        return set_error(L2D_ERR_INVALID, "analyze_addr: bad arguments");
    float thr = 0, nm = 0, fm = 0, sep = 0;
    int st = l2d_kmeans2(lat, n, &thr, &nm, &fm, &sep);
    if (report) {
        report->threshold = thr;
        report->near_cycles = nm;
        report->far_cycles = fm;
        report->separation = sep;
    }
    if (st != L2D_OK) return st;
    // Mask: within each fit page, bit b is active iff line 2^b falls in the other class than
    // the page's first line; bits are then majority-voted over the fit pages.  Pages at index
    // >= num_pages are fit-only pages outside the region (they get no attr entry).
    size_t pages_all = num_pages;
    for (size_t i = 0; i < n; ++i) pages_all = std::max<size_t>(pages_all, (offsets[i] >> kPageShift) + 1);
    std::vector<int> page_base(pages_all, -1);
    std::vector<int> bit_far(pages_all * 32, -1);
    for (size_t i = 0; i < n; ++i) {
        if (kind[i] != 0) continue;
        uint64_t page = offsets[i] >> kPageShift, off = offsets[i] & (kPageBytes - 1);
        int far = lat[i] > thr;
        if (off == 0) page_base[page] = far;
        else if ((off & (off - 1)) == 0) bit_far[page * 32 + __builtin_ctzll(off)] = far;
    }
    int votes[32] = {0}, voters = 0;
    for (size_t p = 0; p < pages_all; ++p) {
        if (page_base[p] < 0) continue;
        ++voters;
        for (int b = kMaskLowBit; b <= kMaskHighBit; ++b) {
            int f = bit_far[p * 32 + b];
            if (f >= 0 && f != page_base[p]) votes[b]++;
        }
    }
    if (voters == 0) return set_error(L2D_ERR_INVALID, "analyze_addr: no mask-fit page");
    uint32_t mask = 0;
    for (int b = kMaskLowBit; b <= kMaskHighBit; ++b)
        if (2 * votes[b] > voters) mask |= 1u << b;
    // attr: every line votes for its page's attr = far xor parity(offset & mask).  A page without
    // any line (a sliver too small to probe) keeps attr 0.
    std::vector<int> ones(pages_all, 0), total(pages_all, 0), attr_all(pages_all, 0);
    for (size_t i = 0; i < n; ++i) {
        uint64_t page = offsets[i] >> kPageShift;
        int v = (lat[i] > thr) ^ (__builtin_popcount(static_cast<uint32_t>(offsets[i]) & mask) & 1);
        ones[page] += v;
        total[page] += 1;
    }
    double worst = 1.0, dom1 = 0.0;
    for (size_t p = 0; p < pages_all; ++p) {
        if (total[p] == 0) continue;
        attr_all[p] = 2 * ones[p] > total[p];
        double agree = static_cast<double>(attr_all[p] ? ones[p] : total[p] - ones[p]) / total[p];
        worst = std::min(worst, agree);
    }
    for (size_t p = 0; p < num_pages; ++p) {
        attr[p] = attr_all[p];
        dom1 += mask ? 0.5 : attr[p];
    }
    // Validation lines: how often the linear model predicts the measured class.
    size_t nval = 0, ok = 0;
    for (size_t i = 0; i < n; ++i) {
        if (kind[i] != 1) continue;
        uint64_t page = offsets[i] >> kPageShift;
        int pred = attr_all[page] ^ (__builtin_popcount(static_cast<uint32_t>(offsets[i]) & mask) & 1);
        ok += pred == static_cast<int>(lat[i] > thr);
        ++nval;
    }
    double magree = nval ? static_cast<double>(ok) / nval : 1.0;
    *mask_out = mask;
    if (report) {
        report->mask = mask;
        report->granule_shift = lowest_bit_or(mask, kPageShift);
        report->mask_agreement = static_cast<float>(magree);
        report->attr_agreement = static_cast<float>(worst);
        report->domain1_fraction = dom1 / static_cast<double>(num_pages);
    }
    if (magree < 0.95)
        return set_error(L2D_ERR_NOT_LINEAR, "linear model (mask 0x%08x) predicts only %.3f of validation lines", mask,
                         magree);
    if (worst < 0.75) return set_error(L2D_ERR_PROBE_AMBIGUOUS, "a page's attr votes agree only %.2f", worst);
    return L2D_OK;
}

// ---- domain-map cache ----------------------------------------------------------------------

}  // extern "C"

namespace {

std::string cache_path(const char *dir, const char *file) {
    std::string p(dir);
    if (!p.empty() && p.back() != '/') p += '/';
    return p + file;
}

}  // namespace

extern "C" {

int l2d_domain_cache_check(const char *dir, const char *key, int num_sm, int *map, int cap, int *num_sm_out,
                           uint32_t *mask) {
    if (!dir || !dir[0] || !num_sm_out) return set_error(L2D_ERR_INVALID, "domain_cache_check: bad arguments");
    if (key) {
        const std::string path = cache_path(dir, "l2d_device.txt");
        FILE *f = std::fopen(path.c_str(), "r");
        if (!f) return set_error(L2D_ERR_STALE, "'%s' missing: the map's device is unknown", path.c_str());
        char buf[L2D_DEVICE_KEY_MAX + 2] = {0};
        const size_t n = std::fread(buf, 1, sizeof buf - 1, f);
        std::fclose(f);
        std::string got(buf, n);
        while (!got.empty() && (got.back() == '\n' || got.back() == '\r')) got.pop_back();
        if (got != key) return set_error(L2D_ERR_STALE, "cache key '%s' differs from this device '%s'", got.c_str(), key);
    }
    int n = 0;
    int st = l2d_read_smid2side_csv(cache_path(dir, "smid2side.csv").c_str(), nullptr, 0, &n);
    if (st != L2D_OK) return st;
    if (num_sm > 0 && n != num_sm)
        return set_error(L2D_ERR_STALE, "cached map has %d SMs, the device has %d", n, num_sm);
    std::vector<int> m(n);
    st = l2d_read_smid2side_csv(cache_path(dir, "smid2side.csv").c_str(), m.data(), n, &n);
    if (st != L2D_OK) return st;
    const int ones = static_cast<int>(std::count(m.begin(), m.end(), 1));
    if (ones == 0 || ones == n) return set_error(L2D_ERR_STALE, "cached map puts every SM in one domain");
    if (mask) {
        st = l2d_read_mask_csv(cache_path(dir, "mask.csv").c_str(), mask);
        if (st != L2D_OK) return st;
    }
    *num_sm_out = n;
    if (map) {
        if (cap < n) return set_error(L2D_ERR_INVALID, "capacity %d < %d SMs", cap, n);
        std::copy(m.begin(), m.end(), map);
    }
    return L2D_OK;
}

int l2d_domain_cache_store(const char *dir, const char *key, const int *map, int num_sm, uint32_t mask) {
    if (!dir || !dir[0] || !key || !map || num_sm <= 0)
        return set_error(L2D_ERR_INVALID, "domain_cache_store: bad arguments");
    if (std::strlen(key) > L2D_DEVICE_KEY_MAX) return set_error(L2D_ERR_INVALID, "device key too long");
    int st = l2d_write_smid2side_csv(cache_path(dir, "smid2side.csv").c_str(), map, num_sm);
    if (st == L2D_OK) st = l2d_write_mask_csv(cache_path(dir, "mask.csv").c_str(), mask);
    if (st != L2D_OK) return st;
    const std::string path = cache_path(dir, "l2d_device.txt");
    FILE *f = std::fopen(path.c_str(), "w");
    if (!f) return set_error(L2D_ERR_IO, "cannot open '%s': %s", path.c_str(), std::strerror(errno));
    std::fprintf(f, "%s\n", key);
    if (std::fclose(f) != 0) return set_error(L2D_ERR_IO, "cannot close '%s'", path.c_str());
    return L2D_OK;
}

}  // extern "C"
