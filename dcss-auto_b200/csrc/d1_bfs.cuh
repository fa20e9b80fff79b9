// Warp-cooperative layered BFS over an 80x70 8-neighbour grid held as bitsets.
//
// Each row is three 32-bit words (bits 0..79 used), 210 words per plane. One BFS
// layer is a 3x3 dilation of the current frontier (a vertical OR of rows y-1..y+1
// followed by a horizontal OR of the +-1 shifts), masked by floor and by the
// not-yet-reached plane. Lane l owns rows l, l+32, l+64. Layered dilation yields
// exactly the FIFO-queue BFS distances of gpu-d1/scripts/learn_env.py:31-39.
#pragma once
#include "d1_common.cuh"

namespace d1 {

constexpr int ROWW = 3, PLANE = H * ROWW;  // 210 words

struct BfsBits {
    uint32_t floor[PLANE], seen[PLANE], cur[PLANE], nxt[PLANE];
};

// Pack a u8[5600] floor map into the row-padded bit plane.
__device__ __forceinline__ void load_floor_bits(const uint8_t *floor, uint32_t *fb, int lane) {
    for (int r = 0; r < PLANE; r++) {
        int y = r / ROWW, x = (r % ROWW) * 32 + lane;
        bool bit = x < W && floor[y * W + x] != 0;
        unsigned b = __ballot_sync(FULL, bit);
        if (lane == 0) fb[r] = b;
    }
    __syncwarp();
}

// Runs layers 1..max_layers from `src`; on_cell(p, k) is called exactly once per
// reached cell (by one lane), k = BFS distance; the source is reported as k = 0.
// stop(k) is evaluated warp-uniformly after layer k and ends the search early.
template <class OnCell, class Stop>
__device__ __forceinline__ int bfs_layers(BfsBits &b, int src, int lane, int max_layers, OnCell on_cell, Stop stop) {
    for (int r = lane; r < PLANE; r += 32) {
        b.seen[r] = 0;
        b.cur[r] = 0;
    }
    __syncwarp();
    if (lane == 0) {
        int r = (src / W) * ROWW + (src % W) / 32;
        uint32_t bit = 1u << ((src % W) % 32);
        b.seen[r] = bit;
        b.cur[r] = bit;
        on_cell(src, 0);
    }
    __syncwarp();
    int k = 1;
    for (; k <= max_layers; k++) {
        if (stop(k - 1)) break;
        bool any = false;
        for (int y = lane; y < H; y += 32) {
            const uint32_t *c0 = b.cur + y * ROWW;
            uint32_t a0 = c0[0], a1 = c0[1], a2 = c0[2];
            if (y > 0) {
                a0 |= c0[-3];
                a1 |= c0[-2];
                a2 |= c0[-1];
            }
            if (y < H - 1) {
                a0 |= c0[3];
                a1 |= c0[4];
                a2 |= c0[5];
            }
            uint32_t d0 = a0 | (a0 << 1) | (a0 >> 1) | (a1 << 31);
            uint32_t d1 = a1 | (a1 << 1) | (a0 >> 31) | (a1 >> 1) | (a2 << 31);
            uint32_t d2 = a2 | (a2 << 1) | (a1 >> 31) | (a2 >> 1);
            const int r = y * ROWW;
            uint32_t n0 = d0 & b.floor[r] & ~b.seen[r];
            uint32_t n1 = d1 & b.floor[r + 1] & ~b.seen[r + 1];
            uint32_t n2 = d2 & b.floor[r + 2] & ~b.seen[r + 2];
            b.nxt[r] = n0;
            b.nxt[r + 1] = n1;
            b.nxt[r + 2] = n2;
            any |= (n0 | n1 | n2) != 0;
        }
        __syncwarp();
        for (int y = lane; y < H; y += 32) {
#pragma unroll
            for (int i = 0; i < ROWW; i++) {
                const int r = y * ROWW + i;
                uint32_t w = b.nxt[r];
                b.seen[r] |= w;
                b.cur[r] = w;
                while (w) {
                    int bit = __ffs(w) - 1;
                    on_cell(y * W + i * 32 + bit, k);
                    w &= w - 1;
                }
            }
        }
        __syncwarp();
        if (!__any_sync(FULL, any)) break;
    }
    return k;
}

template <class OnCell>
__device__ __forceinline__ int bfs_layers(BfsBits &b, int src, int lane, int max_layers, OnCell on_cell) {
    return bfs_layers(b, src, lane, max_layers, on_cell, [](int) { return false; });
}

}  // namespace d1
