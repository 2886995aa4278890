// Shared device helpers for libpbgb200.so (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "pbgb200.h"

namespace pbg {

// ----------------------------------------------------------- error state
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t err, const char* what);
int launch_status(const char* what);
int sm_count();  // streaming multiprocessors of the current device (cached)

#define PBG_REQUIRE(cond, ...)          \
    do {                                \
        if (!(cond)) {                  \
            ::pbg::set_error(__VA_ARGS__); \
            return PBG_EINVAL;          \
        }                               \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Grid for a grid-stride loop: a multiple of the SM count, capped by work.
inline int stride_grid(int64_t items, int block, int blocks_per_sm = 8) {
    int64_t need = (items + block - 1) / block;
    int64_t cap = (int64_t)sm_count() * blocks_per_sm;
    if (need < 1) need = 1;
    return (int)(need < cap ? need : cap);
}

// ------------------------------------------------------------- constants
constexpr int PAD_CARD = 255;
constexpr int LIVE = 0, FOLDED = 1, ALL_IN = 2;
constexpr int FOLD = 0, CHECK_CALL = 1, RAISE_OFFSET = 2;
constexpr int MAXP = 6, MAXD = 52, MAXT = 256;
constexpr uint64_t M63 = 0x7FFFFFFFFFFFFFFFULL;

enum Purpose : int64_t { PRIVATE = 1, ROUND = 2, POSTERIOR = 3, ACTION = 4, CHANCE = 5,
                         COMPLETION = 6, LEARNER = 7, ROLE_SELECTION = 8 };

// ------------------------------------------------------- counter hash
// The v4 counter hash: a 63-bit xor-shift-multiply finaliser.
__host__ __device__ __forceinline__ int64_t mix63(int64_t v) {
    int64_t f = v ^ (v >> 30);
    f = (int64_t)(((uint64_t)f * 0x3C79AC492BA7B653ULL) & M63);
    int64_t s = f ^ (f >> 27);
    s = (int64_t)(((uint64_t)s * 0x1C69B3F74AC4AE35ULL) & M63);
    return (int64_t)((uint64_t)(s ^ (s >> 31)) & M63);
}

__host__ __device__ __forceinline__ uint64_t scalar_hash(uint64_t v) {
    v &= M63;
    v = ((v ^ (v >> 30)) * 0x3C79AC492BA7B653ULL) & M63;
    v = ((v ^ (v >> 27)) * 0x1C69B3F74AC4AE35ULL) & M63;
    return (v ^ (v >> 31)) & M63;
}

// Namespace of (seed, iteration, purpose): computed once on the host, or once per
// row on the device where each row carries its own seed.
__host__ __device__ __forceinline__ uint64_t rng_namespace(int64_t seed, int64_t iteration, int64_t purpose) {
    uint64_t ns = scalar_hash(((uint64_t)seed & M63) ^
                              (((uint64_t)iteration + 0x6A09E667F3BCC909ULL) & M63));
    return scalar_hash(ns ^ (((uint64_t)purpose + 0x5BE0CD19137E2179ULL) & M63));
}

__host__ __device__ __forceinline__ int64_t rng_key(uint64_t ns, int64_t root, int64_t path,
                                                    int64_t draw, int64_t lane, int64_t epoch) {
    uint64_t c = (uint64_t)root * 0x1C69B3F74AC4AE35ULL + (uint64_t)path * 0x3C79AC492BA7B653ULL +
                 (uint64_t)draw * 0x1F83D9ABFB41BD6BULL + (uint64_t)lane * 0x4A7484AA6EA6E483ULL +
                 (uint64_t)epoch * 0x2E1B21385C26C926ULL + ns;
    return mix63((int64_t)(c & M63));
}

__host__ __device__ __forceinline__ int64_t child_path(int64_t path, int64_t ordinal) {
    return mix63(path ^ (int64_t)(((uint64_t)ordinal + 0x243F6A8885A308D3ULL) & M63));
}

// Open-interval fp32 uniform of a key: 24 bits above bit 39, centred.
__device__ __forceinline__ float key_uniform(int64_t key) {
    float mant = (float)((key >> 39) & ((1LL << 24) - 1));
    float u = __fmul_rn(__fadd_rn(mant, 0.5f), 5.9604644775390625e-08f);
    const float top = 0.99999994039535522461f;  // nextafter(1, 0)
    return u < top ? u : top;
}

// --------------------------------------------------------- geometry
struct Geo {
    int P, D, first, H, K, T, E, R;
};

inline Geo derive(pbg_geometry g) {
    Geo d;
    d.P = g.players;
    d.R = g.rank_count;
    d.D = 4 * g.rank_count;
    d.first = 52 - d.D;
    d.H = d.D * (d.D - 1) / 2;
    d.K = g.rank_count * g.rank_count;
    d.T = g.stack_ticks;
    d.E = d.T + 2;
    return d;
}

int check_geometry(pbg_geometry g);

__host__ __device__ __forceinline__ int combo_start(int D, int f) { return f * (2 * D - f - 1) / 2; }

// Inverse of the lexicographic combo id: closed form, then exact fix-up.
__device__ __forceinline__ void combo_cards(int D, int first, int id, int& c0, int& c1) {
    float b = (float)(2 * D - 1);
    int f = (int)((b - sqrtf(fmaxf(b * b - 8.0f * (float)id, 0.0f))) * 0.5f);
    if (f < 0) f = 0;
    if (f > D - 2) f = D - 2;
    while (f < D - 2 && combo_start(D, f + 1) <= id) ++f;
    while (f > 0 && combo_start(D, f) > id) --f;
    c0 = f + first;
    c1 = f + (id - combo_start(D, f)) + 1 + first;
}

__host__ __device__ __forceinline__ int combo_id(int D, int first, int a, int b) {
    int lo = (a < b ? a : b) - first, hi = (a < b ? b : a) - first;
    return lo * (2 * D - lo - 1) / 2 + hi - lo - 1;
}

__device__ __forceinline__ int combo_class(int R, int a, int b) {
    int ra = a / 4 - (13 - R), rb = b / 4 - (13 - R);
    int high = ra > rb ? ra : rb, low = ra > rb ? rb : ra;
    int hp = R - 1 - high, lp = R - 1 - low;
    bool suited_or_pair = (ra == rb) || (a % 4 == b % 4);
    return suited_or_pair ? hp * R + lp : lp * R + hp;
}

// --------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_max_int(int v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_min_int(int v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace pbg
