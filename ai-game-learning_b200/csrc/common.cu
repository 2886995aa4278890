// Error reporting, device properties and the RNG entry points.
#include <string.h>

#include "pbg_common.cuh"

namespace pbg {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int cuda_status(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return PBG_OK;
    set_error("%s: %s", what, cudaGetErrorString(err));
    return PBG_ECUDA;
}

int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

int check_geometry(pbg_geometry g) {
    if (g.players < 2 || g.players > MAXP) { set_error("players must be in [2,6]"); return PBG_EINVAL; }
    if (g.rank_count < 4 || g.rank_count > 13) { set_error("rank_count must be in [4,13]"); return PBG_EINVAL; }
    if (g.stack_ticks < 16 || g.stack_ticks > MAXT) { set_error("stack_ticks must be in [16,256]"); return PBG_EINVAL; }
    if (2 * g.players + 5 >= 4 * g.rank_count) { set_error("NLHE geometry must satisfy 2P+5<4R"); return PBG_EINVAL; }
    return PBG_OK;
}

// rollout.py:122-181
__global__ void keys_kernel(uint64_t ns, int64_t n, const int64_t* root, const int64_t* path, const int64_t* draw,
                            const int64_t* lane, const int64_t* epoch, const uint8_t* active, int64_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t k = rng_key(ns, root[i], path[i], draw[i], lane[i], epoch[i]);
        out[i] = (active && !active[i]) ? 0 : k;
    }
}

__global__ void child_kernel(int64_t n, const int64_t* path, const int64_t* ordinal, int64_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = child_path(path[i], ordinal[i]);
}

__global__ void uniform_kernel(int64_t n, const int64_t* keys, float* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = key_uniform(keys[i]);
}

// rollout.py:237-267, one thread per row: sequential fp32 prefix sum.
__global__ void categorical_kernel(int64_t B, int E, const float* p, const int64_t* keys, const float* mass_in,
                                   int64_t* out) {
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        const float* row = p + b * E;
        float mass = 0.0f;
        if (mass_in) mass = mass_in[b];
        else for (int e = 0; e < E; ++e) mass = __fadd_rn(mass, row[e]);
        float thr = __fmul_rn(key_uniform(keys[b]), mass);
        float cap = nextafterf(mass, 0.0f);
        thr = thr < cap ? thr : cap;
        float cdf = 0.0f;
        int sel = E - 1;
        for (int e = 0; e < E; ++e) {
            cdf = __fadd_rn(cdf, row[e]);
            if (cdf >= thr) { sel = e; break; }
        }
        out[b] = sel;
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" {

const char* pbg_last_error(void) { return g_error; }
int32_t pbg_abi_version(void) { return 1; }

int pbg_rng_keys(int64_t seed, int64_t iteration, int64_t purpose, int64_t n, const int64_t* root,
                 const int64_t* path, const int64_t* draw, const int64_t* lane, const int64_t* epoch,
                 const uint8_t* active, int64_t* out, void* stream) {
    PBG_REQUIRE(purpose > 0, "draw purpose must be a positive namespace identifier");
    PBG_REQUIRE(n >= 0 && root && path && draw && lane && epoch && out, "rng_keys: bad arguments");
    if (n == 0) return PBG_OK;
    keys_kernel<<<stride_grid(n, 256), 256, 0, as_stream(stream)>>>(rng_namespace(seed, iteration, purpose), n, root,
                                                                     path, draw, lane, epoch, active, out);
    return launch_status("rng_keys");
}

int pbg_child_path(int64_t n, const int64_t* path, const int64_t* ordinal, int64_t* out, void* stream) {
    PBG_REQUIRE(n >= 0 && path && ordinal && out, "child_path: bad arguments");
    if (n == 0) return PBG_OK;
    child_kernel<<<stride_grid(n, 256), 256, 0, as_stream(stream)>>>(n, path, ordinal, out);
    return launch_status("child_path");
}

int pbg_logical_uniform(int64_t n, const int64_t* keys, float* out, void* stream) {
    PBG_REQUIRE(n >= 0 && keys && out, "logical_uniform: bad arguments");
    if (n == 0) return PBG_OK;
    uniform_kernel<<<stride_grid(n, 256), 256, 0, as_stream(stream)>>>(n, keys, out);
    return launch_status("logical_uniform");
}

int pbg_logical_categorical(int64_t B, int32_t E, const float* p, const int64_t* keys, const float* mass,
                            int64_t* out, void* stream) {
    PBG_REQUIRE(B >= 0 && E > 0 && p && keys && out, "logical_categorical: bad arguments");
    if (B == 0) return PBG_OK;
    categorical_kernel<<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(B, E, p, keys, mass, out);
    return launch_status("logical_categorical");
}

}  // extern "C"
