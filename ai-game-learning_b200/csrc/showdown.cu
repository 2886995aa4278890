// Sampled-settlement showdown behind the contract-v2 evaluate_showdowns
// signature (called at pbg/games/poker/queued/hooks.py:2277-2295).
//
// The reference delegates ranking to the external poker_gpu_evaluator; this
// kernel ranks 7-card hands directly from rank-multiplicity bit planes and suit
// masks (the board's built once per hand, each seat adding its hole cards),
// with the category order and settlement of showdown.cuh; seats are compared
// through hand_order, whose order is hand_value's (pbg_hand_values exports the
// packed values themselves).
#include "showdown.cuh"

namespace pbg {

__device__ __forceinline__ int64_t hand_value7(const int* cards, const Strength& S, int R) {
    HandCounts h;
    #pragma unroll
    for (int i = 0; i < 7; ++i) h.add(cards[i]);
    return hand_value(h, S, R);
}

__global__ void showdown_kernel(CategoryOrder O, int R, int D, int first, int64_t B, int P, int strata,
                                const uint8_t* board, const int32_t* combo, const int32_t* level,
                                const float* baseline, const float* amount, float* out) {
    // seat loops run over the MAXP slots with an early exit, so the per-seat values stay in registers
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < B; b += (int64_t)gridDim.x * blockDim.x) {
        int64_t value[MAXP];
        int lev[MAXP];
        HandCounts on_board;
        bool board_ok = true;
        #pragma unroll
        for (int i = 0; i < 5; ++i) {
            const int c = board[b * 5 + i];
            board_ok &= c >= first && c < 52;
            if (board_ok) on_board.add(c);
        }
        const int H = D * (D - 1) / 2;
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            value[p] = -1;
            lev[p] = level[b * P + p];
            int id = combo[b * P + p];
            // seats without a valid private combo or board take no share
            if (board_ok && id >= 0 && id < H && lev[p] >= 0) {
                int c0, c1;
                combo_cards(D, first, id, c0, c1);
                HandCounts h = on_board;
                h.add(c0);
                h.add(c1);
                value[p] = hand_order(h, O, R);
            }
        }
        float acc[MAXP];
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            acc[p] = baseline[b * P + p];
        }
        settle_strata(P, strata, value, lev, amount + b * strata, acc);
        #pragma unroll
        for (int p = 0; p < MAXP; ++p) {
            if (p >= P) break;
            out[b * P + p] = acc[p];
        }
    }
}

__global__ void hand_values_kernel(Strength S, int R, int64_t n, const int32_t* cards, int64_t* out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int c[7];
        bool ok = true;
        #pragma unroll
        for (int j = 0; j < 7; ++j) {
            c[j] = cards[i * 7 + j];
            ok &= c[j] >= 0 && c[j] < 52;
        }
        out[i] = ok ? hand_value7(c, S, R) : -1;
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" {

int pbg_evaluate_showdowns(int32_t rank_count, int64_t B, int32_t P, int32_t strata, const uint8_t* board,
                           const int32_t* combo, const int32_t* level, const float* baseline, const float* amount,
                           float* out, void* stream) {
    PBG_REQUIRE(rank_count >= 4 && rank_count <= 13, "evaluate_showdowns: rank_count must be in [4,13]");
    PBG_REQUIRE(P >= 2 && P <= MAXP && strata >= 1 && B >= 0, "evaluate_showdowns: bad shape");
    PBG_REQUIRE(board && combo && level && baseline && amount && out, "evaluate_showdowns: null argument");
    if (B == 0) return PBG_OK;
    int D = 4 * rank_count;
    showdown_kernel<<<stride_grid(B, 128), 128, 0, as_stream(stream)>>>(category_order(rank_count), rank_count, D,
                                                                        52 - D, B, P, strata, board, combo, level,
                                                                        baseline, amount, out);
    return launch_status("evaluate_showdowns");
}

int pbg_hand_values(int32_t rank_count, int64_t n, const int32_t* cards, int64_t* out, void* stream) {
    PBG_REQUIRE(rank_count >= 4 && rank_count <= 13 && n >= 0 && cards && out, "hand_values: bad arguments");
    if (n == 0) return PBG_OK;
    hand_values_kernel<<<stride_grid(n, 128), 128, 0, as_stream(stream)>>>(category_strength(rank_count), rank_count,
                                                                           n, cards, out);
    return launch_status("hand_values");
}

}  // extern "C"
