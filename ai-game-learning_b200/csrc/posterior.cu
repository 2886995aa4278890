// Collision-conditioned posterior profiles for branched Rao-Blackwell poker
// (pbg/games/poker/queued/rb_sampling.py:86-223, sample_children).
//
// Two launches:
//   posterior_cdf_kernel     one warp per (parent, seat), grid-stride; the
//                            hand -> card pair table decoded once per CTA
//                            into shared memory; board-conflicting
//                            private hands weigh 0; the seat's CDF over its
//                            H hands and its mass, accumulated in double and
//                            rounded to fp32 per entry (torch's CPU cumsum);
//                            a warp-wide double scan per 32-hand chunk.
//   posterior_sample_kernel  one warp per child row, lanes = attempts: each
//                            lane draws every seat's hand for its attempt
//                            (POSTERIOR key at draw = attempt, lane = seat;
//                            target = min(u*mass, nextafter(mass, 0)); the
//                            first CDF entry strictly above it: the bucket
//                            from a 32-entry coarse level per seat (loaded
//                            once per row, searched by shuffles), then a
//                            bisection of at most 6 steps inside it, the
//                            seats interleaved so their loads overlap) and
//                            tests the seats' cards for a
//                            collision; a ballot picks the first accepted
//                            attempt of the round, rounds of 32 run until one
//                            succeeds or max_attempts is spent.
// The reference evaluates the whole attempt envelope and takes the first
// success; stopping at the first successful round gives the same profile,
// attempt count and exhaustion flag.  A fresh row whose seat has no
// board-legal mass (the reference's device assert) keeps the inherited
// profile and sets *status = 1 for the host to raise.
#include <climits>

#include "pbg_common.cuh"

namespace pbg {

__device__ __forceinline__ double warp_scan_double(double v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

constexpr int PC_THREADS = 256;
constexpr int PC_MAX_HANDS = 1326;  // 52 cards

// persistent: each CTA decodes the hand -> card pair table into shared memory once, then its warps take
// (parent, seat) rows in a grid stride
__global__ void __launch_bounds__(PC_THREADS)
posterior_cdf_kernel(Geo g, int64_t parents, const float* __restrict__ weights,
                     const uint8_t* __restrict__ board, float* __restrict__ cdf, float* __restrict__ mass) {
    __shared__ uint16_t pair_cards[PC_MAX_HANDS];  // c0 | c1 << 8, absolute card indices
    for (int h = threadIdx.x; h < g.H; h += PC_THREADS) {
        int c0, c1;
        combo_cards(g.D, g.first, h, c0, c1);
        pair_cards[h] = (uint16_t)(c0 | (c1 << 8));
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t rows = parents * g.P;
    const int64_t warps = (int64_t)gridDim.x * (PC_THREADS / 32);
    for (int64_t warp = ((int64_t)blockIdx.x * PC_THREADS + threadIdx.x) >> 5; warp < rows; warp += warps) {
        const int64_t b = warp / g.P;
        uint64_t shown = 0;  // board cards as a 64-bit set (255 = not dealt)
#pragma unroll
        for (int k = 0; k < 5; ++k) {
            const int card = board[b * 5 + k];
            if (card < 64) shown |= 1ull << card;
        }
        const float* w = weights + warp * g.H;
        float* c = cdf + warp * g.H;
        double carry = 0.0;
        // eight 32-hand chunks per group: the group's loads are issued together, so their latency overlaps
        constexpr int GROUP = 8;
        for (int g0 = 0; g0 < g.H; g0 += 32 * GROUP) {
            float loaded[GROUP];
#pragma unroll
            for (int i = 0; i < GROUP; ++i) {
                const int h = g0 + 32 * i + lane;
                loaded[i] = h < g.H ? __ldg(w + h) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < GROUP; ++i) {
                const int h = g0 + 32 * i + lane;
                if (g0 + 32 * i >= g.H) break;
                double v = 0.0;
                if (h < g.H) {
                    const unsigned pc = pair_cards[h];
                    const bool blocked = ((shown >> (pc & 0xffu)) | (shown >> (pc >> 8))) & 1ull;
                    v = blocked ? 0.0 : (double)loaded[i];
                }
                v = warp_scan_double(v, lane) + carry;
                if (h < g.H) c[h] = (float)v;
                carry = __shfl_sync(0xffffffffu, v, 31);
            }
        }
        if (lane == 0) mass[warp] = (float)carry;
    }
}

__global__ void __launch_bounds__(128, 6) posterior_sample_kernel(Geo g, uint64_t ns, int64_t rows, const float* __restrict__ cdf,
                                        const float* __restrict__ mass, const int32_t* __restrict__ inherited,
                                        const int64_t* __restrict__ source, const int64_t* __restrict__ ordinal,
                                        const uint8_t* __restrict__ active, const int64_t* __restrict__ root,
                                        const int64_t* __restrict__ path, const int64_t* __restrict__ epoch,
                                        int64_t epoch_scalar, int max_attempts, int32_t* __restrict__ out,
                                        int32_t* __restrict__ attempt_count, uint8_t* __restrict__ exhausted,
                                        unsigned long long* __restrict__ min_failing, uint32_t* __restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const int P = g.P, H = g.H;
    const int64_t src = source[r];
    const bool fresh = active[r] && ordinal[r] > 0;
    int32_t result = lane < P ? inherited[src * P + lane] : 0;
    int count = 0;
    bool spent = false;
    if (fresh) {
        bool legal = true;
        for (int p = 0; p < P; ++p) legal &= mass[src * P + p] > 0.0f;
        if (!legal) {
            if (lane == 0) atomicOr(status, 1u);
        } else {
            const int64_t rt = root[r], pt = path[r];
            const int64_t ep = epoch ? epoch[r] : epoch_scalar;
            int accepted = -1;
            int32_t mine[MAXP];
            // coarse level of every seat's CDF, loaded once per row: lane j holds the last entry of
            // bucket j (G entries per bucket, 32 buckets cover the H entries)
            const int G = (H + 31) >> 5;
            float coarse[MAXP];
#pragma unroll
            for (int p = 0; p < MAXP; ++p) {
                if (p >= P) break;
                const int idx = (lane + 1) * G - 1;
                coarse[p] = cdf[(src * P + p) * (int64_t)H + (idx < H - 1 ? idx : H - 1)];
            }
            for (int base = 0; base < max_attempts && accepted < 0; base += 32) {
                const int a = base + lane;
                bool ok = a < max_attempts;
                // the seats' bisections advance together, so their dependent CDF loads overlap
                float target[MAXP];
                int lo[MAXP], hi[MAXP];
#pragma unroll
                for (int p = 0; p < MAXP; ++p) {
                    if (p >= P) break;
                    const float total = mass[src * P + p];
                    const float t = __fmul_rn(key_uniform(rng_key(ns, rt, pt, a, p, ep)), total);
                    const float cap = __int_as_float(__float_as_int(total) - 1);  // nextafter(total, 0), total > 0
                    target[p] = cap < t ? cap : t;
                    lo[p] = 0;
                    hi[p] = H;
                }
                // first bucket whose last entry is above the target (a search over the lanes' coarse
                // entries: 33 outcomes, 6 halvings; every lane takes part in every shuffle)
#pragma unroll
                for (int p = 0; p < MAXP; ++p) {
                    if (p >= P) break;
                    int j0 = 0, j1 = 32;
#pragma unroll
                    for (int step = 0; step < 6; ++step) {
                        const int mid = (j0 + j1) >> 1;
                        const float v = __shfl_sync(0xffffffffu, coarse[p], mid & 31);
                        if (j0 < j1) {
                            if (mid < 32 && v <= target[p]) j0 = mid + 1;
                            else j1 = mid;
                        }
                    }
                    // the entry lies in bucket j0 (none above the target: H, clamped below)
                    lo[p] = j0 < 32 ? j0 * G : H;
                    hi[p] = j0 < 32 ? min(j0 * G + G, H) : H;
                }
                // bisection inside the bucket (at most 42 entries at 52 cards: 6 steps), seats interleaved
#pragma unroll
                for (int step = 0; step < 6; ++step) {
#pragma unroll
                    for (int p = 0; p < MAXP; ++p) {
                        if (p >= P) break;
                        if (lo[p] < hi[p]) {
                            const float* c = cdf + (src * P + p) * (int64_t)H;
                            const int mid = (lo[p] + hi[p]) >> 1;
                            if (c[mid] <= target[p]) lo[p] = mid + 1;
                            else hi[p] = mid;
                        }
                    }
                }
                uint64_t held = 0;  // cards of the seats drawn so far; a repeat is a collision
#pragma unroll
                for (int p = 0; p < MAXP; ++p) {
                    if (p >= P) break;
                    mine[p] = lo[p] < H - 1 ? lo[p] : H - 1;
                    int c0, c1;
                    combo_cards(g.D, g.first, mine[p], c0, c1);
                    const uint64_t pair = (1ull << c0) | (1ull << c1);
                    ok &= (held & pair) == 0;
                    held |= pair;
                }
                const unsigned hit = __ballot_sync(0xffffffffu, ok);
                if (hit) {
                    const int winner = __ffs(hit) - 1;
                    accepted = base + winner;
#pragma unroll
                    for (int p = 0; p < MAXP; ++p) {
                        if (p >= P) break;
                        const int32_t v = __shfl_sync(0xffffffffu, mine[p], winner);
                        if (lane == p) result = v;
                    }
                }
            }
            if (accepted >= 0) {
                count = accepted + 1;
            } else {
                count = max_attempts;
                spent = true;
                if (lane == 0) atomicMin(min_failing, (unsigned long long)(pt ^ INT64_MIN));
            }
        }
    }
    if (lane < P) out[r * P + lane] = result;
    if (lane == 0) {
        attempt_count[r] = count;
        exhausted[r] = spent ? 1 : 0;
    }
}

// min_failing is kept as an order-preserving unsigned image (x ^ sign bit) so
// an unsigned atomicMin orders signed paths; this pass turns it back.
__global__ void posterior_finish_kernel(unsigned long long* min_failing) {
    *min_failing = *min_failing ^ (unsigned long long)INT64_MIN;
}

__global__ void posterior_init_kernel(unsigned long long* min_failing) {
    *min_failing = (unsigned long long)INT64_MAX ^ (unsigned long long)INT64_MIN;
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int64_t pbg_posterior_workspace_floats(pbg_geometry geometry, int64_t parents) {
    if (check_geometry(geometry) || parents < 0) return -1;
    const Geo g = derive(geometry);
    return parents * g.P * (int64_t)(g.H + 1);
}

int pbg_posterior_sample_children(pbg_geometry geometry, int64_t parents, const float* range_weights,
                                  const uint8_t* board, const int32_t* inherited, int64_t rows, const int64_t* source,
                                  const int64_t* ordinal, const uint8_t* active, const int64_t* root,
                                  const int64_t* path, int64_t seed, int64_t iteration, const int64_t* retry_epoch,
                                  int64_t retry_epoch_scalar, int32_t max_attempts, float* workspace,
                                  int32_t* profile, int32_t* attempt_count, uint8_t* exhausted, int64_t* min_failing,
                                  uint32_t* status, void* stream) {
    int rc = check_geometry(geometry);
    if (rc) return rc;
    const Geo g = derive(geometry);
    PBG_REQUIRE(parents >= 1 && rows >= 0 && max_attempts >= 1, "posterior: bad sizes");
    // The hand search is a 32-entry coarse level (buckets of G = ceil(H / 32) hands) followed by at
    // most 6 bisection steps inside one bucket, which covers buckets of up to 63 hands: H <= 2016.
    PBG_REQUIRE(g.H <= 2016, "posterior: the coarse level plus 6 bisection steps covers at most 2016 private hands");
    PBG_REQUIRE(range_weights && board && inherited && workspace && min_failing && status,
                "posterior: null pointer");
    PBG_REQUIRE(rows == 0 || (source && ordinal && active && root && path && profile && attempt_count && exhausted),
                "posterior: null row column");
    cudaStream_t s = as_stream(stream);
    float* cdf = workspace;
    float* mass = workspace + parents * g.P * (int64_t)g.H;
    unsigned long long* mf = reinterpret_cast<unsigned long long*>(min_failing);
    posterior_init_kernel<<<1, 1, 0, s>>>(mf);
    posterior_cdf_kernel<<<stride_grid(parents * g.P * 32, PC_THREADS), PC_THREADS, 0, s>>>(g, parents, range_weights,
                                                                                           board, cdf, mass);
    if (rows > 0) {
        const uint64_t ns = rng_namespace(seed, iteration, POSTERIOR);
        const int64_t threads = rows * 32;
        posterior_sample_kernel<<<(unsigned)((threads + 127) / 128), 128, 0, s>>>(
            g, ns, rows, cdf, mass, inherited, source, ordinal, active, root, path, retry_epoch, retry_epoch_scalar,
            max_attempts, profile, attempt_count, exhausted, mf, status);
    }
    posterior_finish_kernel<<<1, 1, 0, s>>>(mf);
    return launch_status("posterior_sample_children");
}

}  // extern "C"
