// compressed-tensors "pack-quantized" words from the library's codes, on the device.
//
// The reference writes only dense fp32 fake-quantised weights (SafetensorsWriter.cs:25-35); the
// checkpoint its documentation names (docs/llm-compressor/deployment.md:124-132) is
// compressed-tensors' pack-quantized layout, whose format is the interface kept here:
//   weight_packed  int32 [m, ceil(n / (32 / bits))]: per element v = q' + 2^(bits-1) in a
//                  bits-wide field, 32 / bits fields per word, first column in the low bits;
//   q'             the signed code: q for a symmetric grid, q - 2^(bits-1) for an asymmetric
//                  one (so v = q + 2^(bits-1) resp. v = q);
//   weight_zero_point (asymmetric, per row or per row and group) int32
//                  [ceil(m / (32 / bits)), G]: zp' + 2^(bits-1) = zp packed along the rows.
// The library's codes are (q - zp) & 0xF nibbles, two per byte with the even column in the high
// nibble (Int4PackedTensor.cs:47-69), for bits <= 4, and the byte q (two's complement when
// symmetric) for bits 5..8; zero-points are int32 per scale entry.
#include "ops.h"

namespace llmc {
namespace {

__device__ __forceinline__ uint32_t code_field(const uint8_t* row, int64_t c, int bits, int sym, int zp) {
    const uint32_t mask = (1u << bits) - 1u;
    if (bits <= 4) {
        const uint8_t b = row[c >> 1];
        const uint32_t nib = (c & 1) ? (b & 0xFu) : (uint32_t)(b >> 4);
        // symmetric: q = the sign-extended nibble, v = q + 2^(bits-1);
        // asymmetric: q = (nibble + zp) mod 16 (q and zp both lie in [0, 2^bits)), v = q.
        if (sym) return (uint32_t)((int)(nib ^ 8u) - 8 + (1 << (bits - 1))) & mask;
        return (nib + (uint32_t)zp) & 0xFu & mask;
    }
    const uint32_t q = row[c];
    return sym ? ((q + (1u << (bits - 1))) & mask) : q;
}

// One thread per packed word.  zrow: zero-point entries per row (0: one shared entry).
__global__ void ct_pack_kernel(const uint8_t* codes, int64_t m, int64_t n, int64_t crow, const int32_t* zps,
                               int64_t zrow, int64_t gs, int bits, int sym, int32_t* out, int64_t ldo) {
    const int per = 32 / bits;
    const int64_t words = (n + per - 1) / per;
    const int64_t total = m * words;
    const bool need_zp = !sym && bits <= 4;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / words, w = t % words;
        const uint8_t* row = codes + r * crow;
        uint32_t word = 0;
        for (int i = 0; i < per; i++) {
            const int64_t c = w * per + i;
            if (c >= n) break;
            const int zp = need_zp ? zps[r * zrow + (zrow > 1 ? c / gs : 0)] : 0;
            word |= code_field(row, c, bits, sym, zp) << (i * bits);
        }
        out[r * ldo + w] = (int32_t)word;
    }
}

// Zero-points zp [m, G] packed along the rows: word (w, g) holds rows w * per .. w * per +
// per - 1, first row in the low bits.
__global__ void ct_pack_zp_kernel(const int32_t* zps, int64_t m, int64_t G, int bits, int32_t* out) {
    const int per = 32 / bits;
    const int64_t words = (m + per - 1) / per;
    const int64_t total = words * G;
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = t / G, g = t % G;
        uint32_t word = 0;
        for (int i = 0; i < per; i++) {
            const int64_t r = w * per + i;
            if (r >= m) break;
            word |= ((uint32_t)zps[r * G + g] & mask) << (i * bits);
        }
        out[w * G + g] = (int32_t)word;
    }
}

int grid_n(llmc_ctx* ctx, int64_t items) {
    int64_t b = (items + 255) / 256;
    const int64_t cap = (int64_t)ctx->sm_count * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

llmc_status ct_pack(llmc_ctx* ctx, const uint8_t* codes, int64_t m, int64_t n, int64_t crow, const int32_t* zps,
                    int64_t zrow, int64_t gs, int bits, int sym, int32_t* out, int64_t ldo, int32_t* zp_out) {
    const int per = 32 / bits;
    const int64_t words = (n + per - 1) / per;
    ct_pack_kernel<<<grid_n(ctx, m * words), 256, 0, ctx->stream>>>(codes, m, n, crow, zps, zrow, gs, bits, sym, out, ldo);
    LLMC_TRY(check_launch(ctx, "ct_pack"));
    if (zp_out) {
        const int64_t zw = (m + per - 1) / per;
        ct_pack_zp_kernel<<<grid_n(ctx, zw * zrow), 256, 0, ctx->stream>>>(zps, m, zrow, bits, zp_out);
        LLMC_TRY(check_launch(ctx, "ct_pack_zp"));
    }
    return LLMC_OK;
}

}  // namespace llmc
