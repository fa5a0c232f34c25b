// synth.cu — seeded synthetic layer inputs.
//
// One counter-based generator serves host and device, so the oracle (host)
// and the device path see identical bytes without copying 0.5 GB per layer:
//   key(seed, stream) and word(key, i) are SplitMix64 finalisers over the
//   counter; bytes are the little-endian bytes of consecutive words.
// Q4_K block b = words [18b, 18b+18) (144 B), then d and dmin (bytes 0..3)
// replaced by fp16(RNE(U(0,0.01))) from a second key. Q6_K block b = first
// 210 bytes of words [27b, 27b+27), with d (bytes 208..209) replaced the same
// way. Every quant and scale byte is thus uniform; Q6_K int8 scales span
// [-128, 127].
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace ofb {

__host__ __device__ inline uint64_t fmix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t gen_key(uint64_t seed, uint64_t stream) {
    return fmix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull +
                  0x632BE59BD9B4E019ull);
}
__host__ __device__ inline uint64_t gen_word(uint64_t key, uint64_t i) {
    return fmix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
}
__host__ __device__ inline double gen_unit(uint64_t w) { return (double)(w >> 11) * 0x1.0p-53; }

// Round-to-nearest-even fp16 bits of a finite v >= 0 (integer-exact steps in
// double, identical on host and device).
__host__ __device__ inline uint16_t half_bits_rne(double v) {
    if (!(v > 0.0)) return 0;
    if (v < 0x1.0p-14) return (uint16_t)rint(v * 0x1.0p24);  // subnormal; 1024 -> min normal
    int e;
    double fr = frexp(v, &e);  // v = fr * 2^e, fr in [0.5, 1)
    double mant = rint((fr * 2.0 - 1.0) * 1024.0);
    int ex = e - 1;
    if (mant >= 1024.0) { mant = 0.0; ex += 1; }
    if (ex > 15) return 0x7C00;
    return (uint16_t)(((ex + 15) << 10) | (int)mant);
}

__host__ __device__ inline uint16_t scale_half(uint64_t key_s, uint64_t i) {
    return half_bits_rne(gen_unit(gen_word(key_s, i)) * 0.01);
}

// Word j (8 bytes) of block b, with the fp16 scale fields folded in.
__host__ __device__ inline uint64_t block_word(int type, uint64_t kq, uint64_t ks, uint64_t b, int j) {
    if (type == OFB_TYPE_Q4_K) {
        uint64_t w = gen_word(kq, b * 18 + j);
        if (j == 0) {
            uint64_t d = scale_half(ks, 2 * b), dm = scale_half(ks, 2 * b + 1);
            w = (w & ~0xFFFFFFFFull) | d | (dm << 16);
        }
        return w;
    }
    uint64_t w = gen_word(kq, b * 27 + j);
    if (j == 26) w = (w & ~0xFFFFull) | scale_half(ks, b);  // bytes 208..209 = d
    return w;
}

__global__ void synth_q4k_kernel(uint64_t *dst, uint64_t n_words, uint64_t first_block,
                                 uint64_t kq, uint64_t ks) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n_words;
         i += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t b = i / 18;
        int j = (int)(i % 18);
        dst[i] = block_word(OFB_TYPE_Q4_K, kq, ks, first_block + b, j);
    }
}

__global__ void synth_q6k_kernel(uint16_t *dst, uint64_t n_blocks, uint64_t first_block,
                                 uint64_t kq, uint64_t ks) {
    uint64_t n = n_blocks * 27;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t b = i / 27;
        int j = (int)(i % 27);
        uint64_t w = block_word(OFB_TYPE_Q6_K, kq, ks, first_block + b, j);
        uint16_t *p = dst + b * (Q6K_BYTES / 2) + j * 4;
        int nh = (j == 26) ? 1 : 4;  // 210 = 26*8 + 2
        for (int h = 0; h < nh; h++) p[h] = (uint16_t)(w >> (16 * h));
    }
}

}  // namespace ofb

using namespace ofb;

extern "C" int ofb_synth_blocks(void *dst, int type, uint64_t n_blocks, uint64_t first_block,
                                uint64_t seed, uint64_t stream_id, void *stream) {
    if (!dst) { set_error("ofb_synth_blocks: NULL dst"); return OFB_EINVAL; }
    uint64_t kq = gen_key(seed, 2 * stream_id), ks = gen_key(seed, 2 * stream_id + 1);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!n_blocks) return OFB_OK;
    if (type == OFB_TYPE_Q4_K) {
        if (reinterpret_cast<uintptr_t>(dst) & 7) { set_error("ofb_synth_blocks: Q4_K dst must be 8-byte aligned"); return OFB_EINVAL; }
        uint64_t nw = n_blocks * 18;
        synth_q4k_kernel<<<grid_for(nw, 256, 148 * 16), 256, 0, s>>>((uint64_t *)dst, nw, first_block, kq, ks);
    } else if (type == OFB_TYPE_Q6_K) {
        if (reinterpret_cast<uintptr_t>(dst) & 1) { set_error("ofb_synth_blocks: Q6_K dst must be 2-byte aligned"); return OFB_EINVAL; }
        synth_q6k_kernel<<<grid_for(n_blocks * 27, 256, 148 * 16), 256, 0, s>>>((uint16_t *)dst, n_blocks, first_block, kq, ks);
    } else {
        set_error("ofb_synth_blocks: type %d is not Q4_K/Q6_K", type);
        return OFB_EINVAL;
    }
    OFB_CHECK_LAUNCH("synth launch");
    return OFB_OK;
}

extern "C" void ofb_synth_blocks_host(void *dst, int type, uint64_t n_blocks, uint64_t first_block,
                                      uint64_t seed, uint64_t stream_id) {
    uint64_t kq = gen_key(seed, 2 * stream_id), ks = gen_key(seed, 2 * stream_id + 1);
    uint8_t *p = static_cast<uint8_t *>(dst);
    const int bytes = (type == OFB_TYPE_Q4_K) ? Q4K_BYTES : Q6K_BYTES;
    const int words = (type == OFB_TYPE_Q4_K) ? 18 : 27;
    for (uint64_t b = 0; b < n_blocks; b++) {
        uint8_t *blk = p + b * bytes;
        for (int j = 0; j < words; j++) {
            uint64_t w = block_word(type, kq, ks, first_block + b, j);
            int nbytes = (8 * j + 8 <= bytes) ? 8 : bytes - 8 * j;
            for (int k = 0; k < nbytes; k++) blk[8 * j + k] = (uint8_t)(w >> (8 * k));
        }
    }
}

extern "C" void ofb_synth_normal_host(float *dst, uint64_t n, uint64_t seed, uint64_t stream_id,
                                      float sigma) {
    uint64_t k = gen_key(seed, 0x4E4F524Dull ^ (stream_id << 1));
    for (uint64_t i = 0; i < n; i++) {
        double u1 = 1.0 - gen_unit(gen_word(k, 2 * i));  // (0, 1]
        double u2 = gen_unit(gen_word(k, 2 * i + 1));
        double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        dst[i] = (float)(z * (double)sigma);
    }
}
