// Device-side view of an s3dsp_hash: the packed 64-bit coordinate key, the
// slot mixer and the linear-probe lookup, shared by the kernels that build
// maps from a hash (kmap.cu) and the coordinate pipeline (coords.cu).
#pragma once

#include "s3dsp_internal.h"

namespace s3dsp {
namespace hash {

constexpr unsigned long long kEmptyKey = ~0ull;

__device__ __forceinline__ bool pack_key(int32_t b, int32_t x, int32_t y, int32_t z,
                                         unsigned long long& key) {
    if ((uint32_t)b > 32767u) return false;
    if (x < -32768 || x > 32767 || y < -32768 || y > 32767 || z < -32768 || z > 32767) return false;
    // b in bits 48..62 (bit 63 clear -> never equals kEmptyKey); the +32768
    // offsets keep the packed order equal to lexicographic (b, x, y, z)
    key = ((unsigned long long)(uint32_t)b << 48) | ((unsigned long long)(uint32_t)(x + 32768) << 32) |
          ((unsigned long long)(uint32_t)(y + 32768) << 16) | (unsigned long long)(uint32_t)(z + 32768);
    return true;
}

__device__ __forceinline__ unsigned long long mix64(unsigned long long k) {
    // 64-bit finaliser (MurmurHash3 fmix64): full avalanche, so spatially
    // clustered keys spread uniformly over the table
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

struct HashView {
    const ulonglong2* slots;
    unsigned long long mask;

    __device__ __forceinline__ int32_t find(unsigned long long key) const {
        unsigned long long s = mix64(key) & mask;
        for (unsigned long long p = 0; p <= mask; ++p) {
            const ulonglong2 kv = __ldg(slots + s);
            if (kv.x == key) return (int32_t)(uint32_t)kv.y;
            if (kv.x == kEmptyKey) return -1;
            s = (s + 1) & mask;
        }
        return -1;
    }
    __device__ __forceinline__ int32_t find_coord(int32_t b, int32_t x, int32_t y, int32_t z) const {
        unsigned long long key;
        if (!pack_key(b, x, y, z, key)) return -1;  // outside the domain -> cannot be present
        return find(key);
    }
};

inline HashView view_of(const s3dsp_hash* h) { return HashView{h->slots, h->capacity - 1}; }

}  // namespace hash
}  // namespace s3dsp
