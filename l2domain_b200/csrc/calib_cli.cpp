// Calibration tools in the reference's file formats, written under $SIDEDGPU_CONFIG_DIR:
//   get_smid2side  -> smid2side.csv   (utility/get_smid2side.cu:114-189: "%d," per SM, newline)
//                     and l2d_device.txt, the key of the device the map was probed on
//   get_mask       -> mask.csv        (utility/get_mask.cu:172-267: "0x%08x"; reads smid2side.csv)
//   get_smid2side --validate: re-probes the SM map and compares it with the cached one (exit 0:
//                     identical; 3: SMs differ; 4: the cache is missing, corrupt or keyed to another
//                     device or driver).  The reference has no validation tool.
// Both probe through libl2d (bounded waits, one cooperative launch); the tool is selected by the
// name it is invoked as (argv[0]) or by the first argument ("smid2side" / "mask").
#include "l2d.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

static std::string config_path(const char *file) {
    const char *dir = std::getenv("SIDEDGPU_CONFIG_DIR");
    if (!dir || !dir[0]) {
        std::fprintf(stderr, "SIDEDGPU_CONFIG_DIR is required\n");
        std::exit(1);
    }
    std::string p(dir);
    if (p.back() != '/') p += '/';
    return p + file;
}

static void die(int st, const char *what) {
    std::fprintf(stderr, "%s failed: %s (%s)\n", what, l2d_status_string(st), l2d_last_error());
    std::exit(1);
}

int main(int argc, char **argv) {
    const char *base = std::strrchr(argv[0], '/');
    base = base ? base + 1 : argv[0];
    bool mask_tool = std::strstr(base, "mask") != nullptr || (argc > 1 && !std::strcmp(argv[1], "mask"));
    int device = 0;
    cudaGetDevice(&device);
    char name[256];
    int num_sm = 0;
    int st = l2d_device_info(device, &num_sm, nullptr, nullptr, nullptr, name, sizeof name);
    if (st) die(st, "device_info");
    std::printf("Device %d: %s has %d SMs\n", device, name, num_sm);
    bool validate = false;
    for (int i = 1; i < argc; ++i) validate |= !std::strcmp(argv[i], "--validate");
    if (!mask_tool && validate) {
        config_path("smid2side.csv");  // requires SIDEDGPU_CONFIG_DIR
        std::vector<int> cached(num_sm), fresh(num_sm);
        int n = 0;
        st = l2d_domain_cache_load(device, std::getenv("SIDEDGPU_CONFIG_DIR"), cached.data(), num_sm, &n, nullptr);
        if (st) {
            std::printf("validate: cache unusable: %s (%s)\n", l2d_status_string(st), l2d_last_error());
            return 4;
        }
        st = l2d_probe_sm_domains(device, fresh.data(), num_sm, &n, nullptr);
        if (st) die(st, "SM probe");
        int diff = 0;
        for (int s = 0; s < num_sm; ++s) diff += cached[s] != fresh[s];
        std::printf("validate: %d of %d SMs differ from the cached map\n", diff, num_sm);
        return diff ? 3 : 0;
    }
    if (!mask_tool) {
        std::vector<int> map(num_sm);
        l2d_sm_probe_report rep{};
        st = l2d_probe_sm_domains_ex(device, map.data(), num_sm, &num_sm, nullptr, &rep, nullptr, 0, nullptr);
        if (st) die(st, "SM probe");
        std::string out = config_path("smid2side.csv");
        st = l2d_write_smid2side_csv(out.c_str(), map.data(), num_sm);
        if (st) die(st, "write smid2side.csv");
        char key[L2D_DEVICE_KEY_MAX + 1];
        st = l2d_device_key(device, key, sizeof key);
        if (st) die(st, "device key");
        std::string kf = config_path("l2d_device.txt");
        FILE *f = std::fopen(kf.c_str(), "w");
        if (!f || std::fprintf(f, "%s\n", key) < 0 || std::fclose(f) != 0) die(L2D_ERR_IO, "write l2d_device.txt");
        std::printf("Elapsed time: %.3f ms\nnear=%.1f far=%.1f cycles, domains %d/%d\n", rep.elapsed_ms,
                    rep.near_cycles, rep.far_cycles, rep.domain_sms[0], rep.domain_sms[1]);
        std::printf("Wrote SMID-to-side map to %s\n", out.c_str());
        return 0;
    }
    std::string in = config_path("smid2side.csv");
    int n = 0;
    st = l2d_read_smid2side_csv(in.c_str(), nullptr, 0, &n);
    if (st) die(st, "read smid2side.csv");
    if (n != num_sm) {
        std::fprintf(stderr, "SMID-to-side map has %d entries, expected %d\n", n, num_sm);
        return 1;
    }
    std::vector<int> map(n);
    st = l2d_read_smid2side_csv(in.c_str(), map.data(), n, &n);
    if (st) die(st, "read smid2side.csv");
    const size_t page = 2ull << 20, bytes = 4 * page;
    void *raw = nullptr;
    if (cudaMalloc(&raw, bytes + page) != cudaSuccess) die(L2D_ERR_CUDA, "cudaMalloc");
    cudaMemset(raw, 0, bytes + page);
    void *mem = reinterpret_cast<void *>((reinterpret_cast<uintptr_t>(raw) + page - 1) & ~(uintptr_t)(page - 1));
    uint32_t mask = 0;
    int attr[4];
    size_t np = 0;
    l2d_addr_probe_report rep{};
    st = l2d_probe_addr_domains_ex(device, mem, bytes, map.data(), n, &mask, attr, 4, &np, nullptr, &rep, nullptr, 0,
                                   nullptr);
    if (st) die(st, "address probe");
    std::string out = config_path("mask.csv");
    st = l2d_write_mask_csv(out.c_str(), mask);
    if (st) die(st, "write mask.csv");
    std::printf("mask = 0x%08x\nElapsed time: %.3f ms\nvalidation agreement %.3f\nWrote mask to %s\n", mask,
                rep.elapsed_ms, rep.mask_agreement, out.c_str());
    cudaFree(raw);
    return 0;
}
