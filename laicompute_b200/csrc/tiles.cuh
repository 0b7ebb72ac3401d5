// Fragment-tile weight layout shared by the matvec kernels, the embedding
// gather and the upload repack.
//
// A matrix of R rows x K columns (GGUF blocks of 32 columns) is cut into
// tile-blocks of 16 rows x 32 columns. Tile-blocks are stored tile-major
// ([row tile][block]) so the blocks of one row tile form one contiguous run.
// Inside a tile-block, lane L = 4g + c of a warp owns rows g and g+8 and
// columns 8c..8c+7 — exactly its A-operand fragment of mma.m16n8k16:
//   Q4_0  8 bytes per lane: 4 nibble bytes of row g, 4 of row g+8 (file order)
//   Q8_0 16 bytes per lane: 8 int8 of row g, 8 of row g+8 (fragment order)
//   F16  32 bytes per lane: 8 binary16 of row g, 8 of row g+8 (fragment order)
// and the 16 binary16 block scales sit in a separate 32-byte record per
// tile-block as (row g, row g+8) pairs. Fragment order of an 8-column group
// is 0,4,1,5,2,6,3,7 so that columns (k, k+4) share one half2 register.
#pragma once
#include "common.cuh"

namespace laic {

// bytes of one 16x32 tile-block of quants (per type) and of its scales
__host__ __device__ constexpr int tile_qbytes(int type) { return type == T_Q4_0 ? 256 : type == T_Q8_0 ? 512 : 1024; }
constexpr int kTileSBytes = 32;

// Position of column k (0..7) of an 8-column group inside its lane fragment.
__host__ __device__ constexpr int frag_pos(int k) { return k < 4 ? 2 * k : 2 * (k - 4) + 1; }


// Byte offset of element (row r, col i) in the quant plane, and of its scale.
__host__ __device__ __forceinline__ size_t tile_elem_offset(int type, int nb, int r, int i) {
    const int t = r >> 4, rr = r & 15, g = rr & 7, h = rr >> 3;
    const int b = i >> 5, o = i & 31, cc = o >> 3, k = o & 7;
    const size_t chunk = ((size_t)t * nb + b) * tile_qbytes(type);
    const int L = g * 4 + cc;
    if (type == T_Q4_0) return chunk + L * 8 + h * 4 + (k >> 1);
    if (type == T_Q8_0) return chunk + L * 16 + h * 8 + frag_pos(k);
    return chunk + L * 32 + h * 16 + frag_pos(k) * 2;
}
__host__ __device__ __forceinline__ size_t tile_scale_offset(int nb, int r, int b) {
    const int t = r >> 4, rr = r & 15;
    return ((size_t)t * nb + b) * kTileSBytes + (rr & 7) * 4 + (rr >> 3) * 2;
}

// One element, decoded exactly as quant_v2::value / GgufTensor::value.
__device__ __forceinline__ float tile_value(int type, const uint8_t* q, const uint8_t* s, int nb, int r, int i) {
    const size_t off = tile_elem_offset(type, nb, r, i);
    if (type == T_F16) return __half2float(*reinterpret_cast<const __half*>(q + off));
    const float d = __half2float(*reinterpret_cast<const __half*>(s + tile_scale_offset(nb, r, i >> 5)));
    if (type == T_Q8_0) return d * float((int8_t)q[off]);
    const uint8_t z = q[off];
    return d * float((((i & 31) & 1) ? (z >> 4) : (z & 15)) - 8);
}

// GGUF rows -> fragment tiles. Source row r of the chunk lands in matrix row
// r*row_mul + row_add (row_mul 2 interleaves the gate and up matrices).
static __global__ void repack_tiles_kernel(int type, const uint8_t* __restrict__ src, long long rows, int nb, int row_mul,
                                    long long row_add, uint8_t* __restrict__ q, uint8_t* __restrict__ s) {
    const long long total = rows * nb;
    const int sbb = type == T_F16 ? 64 : type == T_Q4_0 ? 18 : 34;  // source bytes per 32 elements
    for (long long blk = blockIdx.x * (long long)blockDim.x + threadIdx.x; blk < total;
         blk += (long long)gridDim.x * blockDim.x) {
        const long long r = blk / nb;
        const int b = (int)(blk % nb);
        const int dr = (int)(r * row_mul + row_add);
        const uint8_t* sp = src + blk * sbb;
        if (type == T_F16) {
            for (int o = 0; o < 32; ++o) {
                const size_t off = tile_elem_offset(type, nb, dr, b * 32 + o);
                q[off] = sp[2 * o];
                q[off + 1] = sp[2 * o + 1];
            }
            continue;
        }
        const size_t so = tile_scale_offset(nb, dr, b);
        s[so] = sp[0];
        s[so + 1] = sp[1];
        if (type == T_Q8_0) {
            for (int o = 0; o < 32; ++o) q[tile_elem_offset(type, nb, dr, b * 32 + o)] = sp[2 + o];
        } else {
            for (int j = 0; j < 16; ++j) q[tile_elem_offset(type, nb, dr, b * 32 + 2 * j)] = sp[2 + j];
        }
    }
}

static __global__ void tile_dequant_kernel(int type, const uint8_t* q, const uint8_t* s, int in, int nb, long long rows,
                                    float* out) {
    const long long total = rows * in;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x)
        out[e] = tile_value(type, q, s, nb, (int)(e / in), (int)(e % in));
}

}  // namespace laic
