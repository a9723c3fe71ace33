// pack.cuh - one-time repack of the reference's Q4_0 expert tensors into device planes.
//
// Input: the GGUF layout bound by runtime/src/model.rs:36-40 - per expert, gate_up is 2*ff rows
// (gate rows 0..ff-1, then up rows) of n_embd/32 18-byte blocks; down is n_embd rows of ff/32
// blocks. The HIP executor uploads these bytes unchanged (runtime/src/hip_exec.rs:429-433);
// this backend splits each block into a 16-byte nibble plane and an f16 scale plane (so every
// copy is 16-byte aligned for TMA and every row of nibbles is one contiguous run), and
// interleaves gate and up rows per 32 columns:
//   packed gate_up row R = q*64 + s*32 + i  holds  original row s*ff + q*32 + i,
// and within a packed row R (gate_up or down) the 16-byte nibble block b sits at position
// nib_pos(b) = b ^ (R & 7) when b lies in a complete group of 8 blocks, at b otherwise (the
// tail of a down row: 22 blocks per row for ff = 704), so that threads reading block b of 8
// consecutive rows hit distinct shared-memory banks. Gate_up rows hold a multiple of 8
// blocks. Scales are not swizzled.
// The prefill GEMM reads the scales a third time, as f32 in a tile-major plane: 128-row tiles
// of packed rows, per tile [block][row] (one block's scales of a tile are 512 contiguous bytes,
// a stage's copy a single bulk transfer). Rows are padded up to a multiple of 128.
// Nibble bytes and scale bits are copied unchanged (the f32 scales are the f16 values exactly),
// so every dot product sees the same integers and scales as the reference.
#pragma once
#include "common.cuh"

namespace rvc {

// Packed expert planes (byte offsets inside the packed buffer are computed on the host).
struct PackedView {
    const uint8_t *gu_nib;   // [E][2*ff packed rows][nb][16]
    const uint16_t *gu_scl;  // [E][2*ff][nb]
    const uint8_t *dn_nib;   // [E][n_embd][nbh][16]
    const uint16_t *dn_scl;  // [E][n_embd][nbh]
    const float *gu_dw;      // [E * 2*ff / 128][nb][128] f32
    const float *dn_dw;      // [E * n_embd / 128][nbh][128] f32
};

constexpr int DW_TILE = 128;  // rows per tile of the f32 scale planes

// Position of nibble block b in a packed row of nblk blocks whose row index has low bits key.
__host__ __device__ __forceinline__ int nib_pos(int b, int nblk, int key) { return b < (nblk & ~7) ? (b ^ key) : b; }

__global__ void k_pack_q4(const uint8_t *__restrict__ src, int n_experts, int rows, int nblk, bool interleave_gu,
                          int ff, uint8_t *__restrict__ nib, uint16_t *__restrict__ scl) {
    const size_t total = (size_t)n_experts * rows * nblk;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t b = i % nblk;
        const size_t row = (i / nblk) % rows;
        const size_t e = i / ((size_t)nblk * rows);
        size_t prow = row;
        if (interleave_gu) {
            const size_t s = row / ff, col = row % ff;
            prow = (col / 32) * 64 + s * 32 + (col % 32);
        }
        const uint8_t *blk = src + i * Q4_BLOCK;
        const size_t dst = (e * rows + prow) * nblk + b;
        const size_t dnib = (e * rows + prow) * nblk + nib_pos((int)b, nblk, (int)(prow & 7));
        // 18-byte blocks are only 2-byte aligned: read as 9 halfwords
        const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = (uint32_t)h[1 + 2 * j] | ((uint32_t)h[2 + 2 * j] << 16);
        *reinterpret_cast<uint4 *>(nib + dnib * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        scl[dst] = h[0];
    }
}

// The f32 tile-major scale plane from the packed f16 plane [E * rows][nblk] (rows per expert a
// multiple of DW_TILE, so no tile straddles two experts).
__global__ void k_pack_dw(const uint16_t *__restrict__ scl, size_t n_rows, int nblk, float *__restrict__ dw) {
    const size_t total = n_rows * nblk;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i % DW_TILE, b = (i / DW_TILE) % nblk, t = i / ((size_t)DW_TILE * nblk);
        dw[i] = f16_bits_to_f32(scl[(t * DW_TILE + r) * nblk + b]);
    }
}

}  // namespace rvc
