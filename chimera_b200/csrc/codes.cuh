// Packed (1..8)-bit code layouts of rabitqlib's packing_rabitqplus_code
// (cpp/third_party/rabitqlib/quantization/pack_excode.hpp:13-297), written
// as per-dimension / per-byte formulas usable on host and device.
//
// code_at(p, i, w):      value of dimension i in a packed 128-dim code.
// packed_byte(raw, b, w): byte b of the packed code of 128 raw values.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define CHM_HD __host__ __device__ __forceinline__
#else
#define CHM_HD inline
#endif

namespace chm {

CHM_HD int code_at(const uint8_t* p, int i, int w) {
    switch (w) {
        case 1: return (p[2 * (i >> 4) + ((i & 15) >> 3)] >> (i & 7)) & 1;
        case 2: return (p[4 * (i >> 4) + (i & 3)] >> (2 * ((i & 15) >> 2))) & 3;
        case 3: {
            const uint8_t* g = p + 24 * (i >> 6);
            const int r = i & 63;
            return ((g[r & 15] >> (2 * (r >> 4))) & 3) | (((g[16 + (r & 7)] >> (r >> 3)) & 1) << 2);
        }
        case 4: return (p[8 * (i >> 4) + (i & 7)] >> (4 * ((i & 15) >> 3))) & 15;
        case 5: {
            const uint8_t* g = p + 40 * (i >> 6);
            const int r = i & 63;
            const int lo = (g[16 * (r >> 5) + (r & 15)] >> (4 * ((r >> 4) & 1))) & 15;
            return lo | (((g[32 + (r & 7)] >> (r >> 3)) & 1) << 4);
        }
        case 6: {
            const uint8_t* g = p + 12 * (i >> 4);
            const int j = i & 15;
            return ((g[j & 7] >> (4 * (j >> 3))) & 15) | (((g[8 + (j & 3)] >> (2 * (j >> 2))) & 3) << 4);
        }
        case 7: {
            const uint8_t* g = p + 56 * (i >> 6);
            const int r = i & 63;
            int lo;
            if (r < 48) {
                lo = g[r] & 63;
            } else {
                const int j = r - 48;
                lo = ((g[j] >> 6) & 3) | (((g[16 + j] >> 6) & 3) << 2) | (((g[32 + j] >> 6) & 3) << 4);
            }
            return lo | (((g[48 + (r & 7)] >> (r >> 3)) & 1) << 6);
        }
        default: return p[i];
    }
}

CHM_HD uint8_t packed_byte(const uint8_t* raw, int b, int w) {
    int v = 0;
    switch (w) {
        case 1: {
            const int base = 16 * (b >> 1) + 8 * (b & 1);
            for (int j = 0; j < 8; ++j) v |= (raw[base + j] & 1) << j;
            break;
        }
        case 2: {
            const int base = 16 * (b >> 2), j = b & 3;
            for (int s = 0; s < 4; ++s) v |= (raw[base + 4 * s + j] & 3) << (2 * s);
            break;
        }
        case 3: {
            const int g = 64 * (b / 24), r = b % 24;
            if (r < 16) {
                for (int s = 0; s < 4; ++s) v |= (raw[g + 16 * s + r] & 3) << (2 * s);
            } else {
                const int k = r - 16;
                for (int m = 0; m < 8; ++m) v |= ((raw[g + 8 * m + k] >> 2) & 1) << m;
            }
            break;
        }
        case 4: {
            const int base = 16 * (b >> 3), k = b & 7;
            v = (raw[base + k] & 15) | ((raw[base + 8 + k] & 15) << 4);
            break;
        }
        case 5: {
            const int g = 64 * (b / 40), r = b % 40;
            if (r < 32) {
                const int base = g + 32 * (r >> 4), j = r & 15;
                v = (raw[base + j] & 15) | ((raw[base + 16 + j] & 15) << 4);
            } else {
                const int k = r - 32;
                for (int m = 0; m < 8; ++m) v |= ((raw[g + 8 * m + k] >> 4) & 1) << m;
            }
            break;
        }
        case 6: {
            const int base = 16 * (b / 12), r = b % 12;
            if (r < 8) {
                v = (raw[base + r] & 15) | ((raw[base + 8 + r] & 15) << 4);
            } else {
                const int k = r - 8;
                for (int s = 0; s < 4; ++s) v |= ((raw[base + 4 * s + k] >> 4) & 3) << (2 * s);
            }
            break;
        }
        case 7: {
            const int g = 64 * (b / 56), r = b % 56;
            if (r < 48) {
                const int vec = r >> 4, j = r & 15;
                v = (raw[g + 16 * vec + j] & 63) | (((raw[g + 48 + j] >> (2 * vec)) & 3) << 6);
            } else {
                const int k = r - 48;
                for (int m = 0; m < 8; ++m) v |= ((raw[g + 8 * m + k] >> 6) & 1) << m;
            }
            break;
        }
        default: v = raw[b];
    }
    return (uint8_t)v;
}

}  // namespace chm
