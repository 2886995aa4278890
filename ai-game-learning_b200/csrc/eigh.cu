// Batched symmetric eigendecomposition for small matrices (n <= 64): the
// cyclic Jacobi method (C. G. J. Jacobi, 1846) with the parallel round-robin
// ordering of Brent & Luk (1985), one CTA per matrix, in fp32.
//
// The multiway folded statistics diagonalise one beta matrix per decision
// (pbg/games/poker/queued/folded.py:352, torch.linalg.eigh of [B, C, C] with
// C = 52 at R13); a library call handles such a batch one matrix at a time.
// Here a CTA holds its matrix A and the accumulated rotations V in shared
// memory.  A sweep visits every index pair once in n' - 1 rounds (n' = n
// rounded up to even; a padding index pairs with nothing); the n'/2 pairs of a
// round are disjoint, so their rotations are computed together (one thread per
// pair: t = sign(tau) / (|tau| + sqrt(1 + tau^2)), tau = (a_qq - a_pp) / 2 a_pq,
// c = 1 / sqrt(1 + t^2), s = t c, the rotation that zeroes a_pq) and applied
// together: A <- J^T A (rows p, q), then A <- A J and V <- V J (columns p, q);
// the pairs of a round follow the circle method in closed form.  Sweeps stop
// when the off-diagonal mass reaches the fp32 floor, or stops falling once it
// is near that floor (or after the given number of sweeps).  Eigenvalues are the diagonal, eigenvectors the
// columns of V, unsorted.
#include "pbg_common.cuh"

namespace pbg {

constexpr int EJ_MAXN = 64;
constexpr int EJ_LD = EJ_MAXN + 1;  // padded row stride (bank spread)
constexpr int EJ_THREADS = 256;

// pair k of round r of the circle method over `even` indices (p < q)
__device__ __forceinline__ void ej_pair(int even, int r, int k, int& p, int& q) {
    const int m = even - 1;
    if (k == 0) {
        p = r;
        q = m;
    } else {
        p = (r + k) % m;
        q = (r - k + m) % m;
    }
    if (p > q) {
        const int t = p;
        p = q;
        q = t;
    }
}

__global__ void __launch_bounds__(EJ_THREADS)
jacobi_eigh_kernel(int n, const float* __restrict__ matrices, float* __restrict__ values, float* __restrict__ vectors,
                   int max_sweeps) {
    __shared__ float A[EJ_MAXN * EJ_LD];
    __shared__ float V[EJ_MAXN * EJ_LD];
    __shared__ float cs[EJ_MAXN / 2][2];
    __shared__ int pairs[EJ_MAXN / 2][2];
    __shared__ float norms[2];
    const int64_t m = blockIdx.x;
    const float* src = matrices + m * (int64_t)n * n;
    const int even = (n + 1) & ~1;
    const int half = even / 2;
    for (int i = threadIdx.x; i < n * n; i += EJ_THREADS) {
        const int r = i / n, c = i - r * n;
        A[r * EJ_LD + c] = 0.5f * (src[r * n + c] + src[c * n + r]);  // symmetric part, as eigh reads one triangle
        V[r * EJ_LD + c] = r == c ? 1.0f : 0.0f;
    }
    __syncthreads();
    float previous_off = INFINITY;
    for (int sweep = 0; sweep < max_sweeps; ++sweep) {
        // convergence: off-diagonal against total squared mass
        if (threadIdx.x < 32) {
            float off = 0.0f, total = 0.0f;
            for (int i = threadIdx.x; i < n * n; i += 32) {
                const int r = i / n, c = i - r * n;
                const float a = A[r * EJ_LD + c];
                total += a * a;
                if (r != c) off += a * a;
            }
            off = warp_sum(off);
            total = warp_sum(total);
            if (threadIdx.x == 0) {
                norms[0] = off;
                norms[1] = total;
            }
        }
        __syncthreads();
        // converged: the off-diagonal mass is at the fp32 floor (1e-12 of the total), or it is small
        // (1e-9 of the total, where convergence is quadratic) and the last sweep removed less than three
        // quarters of it (rounding floor reached).  Early sweeps converge only linearly, by 3-5x each.
        const float off = norms[0];
        if (!(off > 1e-12f * norms[1]) || (off <= 1e-9f * norms[1] && off > 0.25f * previous_off)) break;
        previous_off = off;
        for (int round = 0; round < even - 1; ++round) {
            // round-robin (circle) pairing: index even-1 fixed, pair k of round r joins
            // (r + k) mod (even-1) and (r - k) mod (even-1), pair 0 joins r with the fixed index
            if (threadIdx.x < half) {
                const int k = threadIdx.x;
                int p, q;
                ej_pair(even, round, k, p, q);
                float c = 1.0f, s = 0.0f;
                if (q < n) {
                    const float apq = A[p * EJ_LD + q];
                    if (apq != 0.0f) {
                        const float tau = (A[q * EJ_LD + q] - A[p * EJ_LD + p]) / (2.0f * apq);
                        const float t = copysignf(1.0f, tau) / (fabsf(tau) + sqrtf(1.0f + tau * tau));
                        c = rsqrtf(1.0f + t * t);
                        s = t * c;
                    }
                }
                cs[k][0] = c;
                cs[k][1] = s;
                pairs[k][0] = p;
                pairs[k][1] = q;
            }
            __syncthreads();
            // rows p, q of A: A <- J^T A.  Thread t owns column t mod 64 for the pairs k = t / 64 (mod 4).
            const int lane64 = threadIdx.x & (EJ_MAXN - 1), group = threadIdx.x / EJ_MAXN;
            constexpr int GROUPS = EJ_THREADS / EJ_MAXN;
            if (lane64 < n) {
                const int col = lane64;
                for (int k = group; k < half; k += GROUPS) {
                    const int p = pairs[k][0], q = pairs[k][1];
                    if (q >= n) continue;
                    const float c = cs[k][0], s = cs[k][1];
                    const float ap = A[p * EJ_LD + col], aq = A[q * EJ_LD + col];
                    A[p * EJ_LD + col] = c * ap - s * aq;
                    A[q * EJ_LD + col] = s * ap + c * aq;
                }
            }
            __syncthreads();
            // columns p, q of A and V: A <- A J, V <- V J (thread t owns row t mod 64)
            for (int k = group; k < half && lane64 < n; k += GROUPS) {
                const int row = lane64;
                const int p = pairs[k][0], q = pairs[k][1];
                if (q >= n) continue;
                const float c = cs[k][0], s = cs[k][1];
                const float ap = A[row * EJ_LD + p], aq = A[row * EJ_LD + q];
                A[row * EJ_LD + p] = c * ap - s * aq;
                A[row * EJ_LD + q] = s * ap + c * aq;
                const float vp = V[row * EJ_LD + p], vq = V[row * EJ_LD + q];
                V[row * EJ_LD + p] = c * vp - s * vq;
                V[row * EJ_LD + q] = s * vp + c * vq;
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += EJ_THREADS) values[m * n + i] = A[i * EJ_LD + i];
    for (int i = threadIdx.x; i < n * n; i += EJ_THREADS) {
        const int r = i / n, c = i - r * n;
        vectors[m * (int64_t)n * n + i] = V[r * EJ_LD + c];
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_symmetric_eigh(int64_t batch, int32_t n, const float* matrices, float* values, float* vectors,
                                  int32_t max_sweeps, void* stream) {
    PBG_REQUIRE(batch >= 0 && batch <= INT32_MAX, "symmetric_eigh: bad batch");
    PBG_REQUIRE(n >= 1 && n <= EJ_MAXN, "symmetric_eigh: n must be in [1, 64]");
    PBG_REQUIRE(max_sweeps >= 1 && max_sweeps <= 64, "symmetric_eigh: sweeps must be in [1, 64]");
    if (batch == 0) return PBG_OK;
    PBG_REQUIRE(matrices && values && vectors, "symmetric_eigh: null pointer");
    jacobi_eigh_kernel<<<(unsigned)batch, EJ_THREADS, 0, as_stream(stream)>>>(n, matrices, values, vectors,
                                                                               max_sweeps);
    return launch_status("symmetric_eigh");
}
