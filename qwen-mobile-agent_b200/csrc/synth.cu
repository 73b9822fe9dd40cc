// synth.cu -- on-device synthetic weights for random-init qwen35moe models.
//
// Every tensor value is a pure function of (seed, tensor name, element
// index): an Irwin-Hall(4) normal from one splitmix64 hash, scaled by the
// tensor's kind, then quantized by the engine's Q4_K / Q6_K / Q8_0
// quantizers.  The arithmetic is written with explicit round-to-nearest
// intrinsics (no fused multiply-add), IEEE division and roundf, so the bytes
// equal those of the CPU generator the tests use as their oracle.  The
// reference ships no quantizer (its weights come from a GGUF file), so this
// is the engine's own definition of "weights ~N(0,0.02) then quantized".
#include <string.h>

#include "common.cuh"
#include "synth.cuh"

namespace qma {

uint64_t name_key(const char *name, uint64_t seed) {
    uint64_t h = 0xcbf29ce484222325ull;   // FNV-1a 64
    for (const char *p = name; *p; p++) {
        h ^= uint8_t(*p);
        h *= 0x100000001b3ull;
    }
    return h ^ (seed * 0x9E3779B97F4A7C15ull);
}

int tensor_kind(const char *name) {
    const size_t n = strlen(name);
    const char *sfx = "norm.weight";
    const size_t ls = strlen(sfx);
    if (n >= ls && strcmp(name + n - ls, sfx) == 0) return KIND_NORM;
    if (strstr(name, "ssm_conv1d")) return KIND_CONV;
    if (strstr(name, "ssm_dt")) return KIND_DT;
    if (n >= 5 && strcmp(name + n - 5, "ssm_a") == 0) return KIND_A;
    return KIND_W;
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t idx) {
    const uint64_t h = splitmix64(key + idx);
    const int s = int(h & 0xffff) + int((h >> 16) & 0xffff) + int((h >> 32) & 0xffff) + int(h >> 48);
    return __fmul_rn(__int2float_rn(s - 131070), 0x1.bb67aep-16f);
}

__device__ __forceinline__ float kind_value(int kind, uint64_t key, uint64_t idx) {
    const float v = synth_normal(key, idx);
    switch (kind) {
    case KIND_NORM: return __fadd_rn(1.0f, __fmul_rn(0.05f, v));
    case KIND_CONV: return __fadd_rn(0.0f, __fmul_rn(0.25f, v));
    case KIND_DT: return __fadd_rn(0.0f, __fmul_rn(0.5f, v));
    case KIND_A: return __fsub_rn(-0.5f, __fmul_rn(0.25f, fabsf(v)));
    default: return __fadd_rn(0.0f, __fmul_rn(0.02f, v));
    }
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ uint16_t f2h(float x) { return __half_as_ushort(__float2half_rn(x)); }

// Q4_K quantizer (same steps as the oracle's qo_quantize_q4k)
__device__ void quantize_q4k(const float *x, uint8_t *blk) {
    float scale[8], mins[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int i = 1; i < 32; i++) {
            const float v = x[32 * j + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        mins[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const uint16_t dh = f2h(__fdiv_rn(max_scale, 63.0f));
    const uint16_t mh = f2h(__fdiv_rn(max_min, 63.0f));
    const float dq = h2f(dh), mq = h2f(mh);
    uint8_t sc[8], mm[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = uint8_t(dq > 0.0f ? clampi(int(roundf(__fdiv_rn(scale[j], dq))), 0, 63) : 0);
        mm[j] = uint8_t(mq > 0.0f ? clampi(int(roundf(__fdiv_rn(mins[j], mq))), 0, 63) : 0);
    }
    blk[0] = uint8_t(dh & 0xff); blk[1] = uint8_t(dh >> 8);
    blk[2] = uint8_t(mh & 0xff); blk[3] = uint8_t(mh >> 8);
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = uint8_t((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = uint8_t((mm[j] & 63) | ((mm[j + 4] >> 4) << 6));
        s[j + 8] = uint8_t((sc[j + 4] & 0xF) | ((mm[j + 4] & 0xF) << 4));
    }
    uint8_t *qs = blk + 16;
    for (int g = 0; g < 4; g++) {
        const int j0 = 2 * g, j1 = 2 * g + 1;
        const float ds0 = __fmul_rn(dq, float(sc[j0])), dm0 = __fmul_rn(mq, float(mm[j0]));
        const float ds1 = __fmul_rn(dq, float(sc[j1])), dm1 = __fmul_rn(mq, float(mm[j1]));
        const float id0 = ds0 > 0.0f ? __fdiv_rn(1.0f, ds0) : 0.0f;
        const float id1 = ds1 > 0.0f ? __fdiv_rn(1.0f, ds1) : 0.0f;
        for (int l = 0; l < 32; l++) {
            const int q0 = ds0 > 0.0f ? clampi(int(roundf(__fmul_rn(__fadd_rn(x[32 * j0 + l], dm0), id0))), 0, 15) : 0;
            const int q1 = ds1 > 0.0f ? clampi(int(roundf(__fmul_rn(__fadd_rn(x[32 * j1 + l], dm1), id1))), 0, 15) : 0;
            qs[32 * g + l] = uint8_t(q0 | (q1 << 4));
        }
    }
}

// Q6_K quantizer (qo_quantize_q6k)
__device__ void quantize_q6k(const float *x, uint8_t *blk) {
    float scale[16];
    float max_scale = 0.0f;
    for (int g = 0; g < 16; g++) {
        float amax = 0.0f;
        for (int i = 0; i < 16; i++) {
            const float a = fabsf(x[16 * g + i]);
            if (a > amax) amax = a;
        }
        scale[g] = __fdiv_rn(amax, 31.0f);
        if (scale[g] > max_scale) max_scale = scale[g];
    }
    const uint16_t dh = f2h(__fdiv_rn(max_scale, 127.0f));
    const float dq = h2f(dh);
    for (int k = 0; k < 192; k++) blk[k] = 0;
    for (int g = 0; g < 16; g++) {
        const int sc = dq > 0.0f ? clampi(int(roundf(__fdiv_rn(scale[g], dq))), -128, 127) : 0;
        blk[192 + g] = uint8_t(int8_t(sc));
        const float ds = __fmul_rn(dq, float(sc));
        const float ids = ds > 0.0f ? __fdiv_rn(1.0f, ds) : 0.0f;
        for (int i = 0; i < 16; i++) {
            const int q = ds > 0.0f ? clampi(int(roundf(__fmul_rn(x[16 * g + i], ids))), -32, 31) : 0;
            const int v = q + 32;
            const int w = (16 * g + i) & 127, half = (16 * g + i) >> 7;
            const int L = w & 63, hi = w >> 6;
            const int shift = 2 * ((L >> 5) + 2 * hi);
            if (hi) blk[64 * half + L] |= uint8_t((v & 0xF) << 4);
            else blk[64 * half + L] |= uint8_t(v & 0xF);
            blk[128 + 32 * half + (L & 31)] |= uint8_t(((v >> 4) & 3) << shift);
        }
    }
    blk[208] = uint8_t(dh & 0xff);
    blk[209] = uint8_t(dh >> 8);
}

// Q8_0 quantizer (qo_quantize_q80)
__device__ void quantize_q80(const float *x, uint8_t *blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
        const float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    const uint16_t dh = f2h(__fdiv_rn(amax, 127.0f));
    const float dq = h2f(dh);
    const float id = dq > 0.0f ? __fdiv_rn(1.0f, dq) : 0.0f;
    blk[0] = uint8_t(dh & 0xff);
    blk[1] = uint8_t(dh >> 8);
    for (int i = 0; i < 32; i++) blk[2 + i] = uint8_t(int8_t(clampi(int(roundf(__fmul_rn(x[i], id))), -127, 127)));
}

// One thread per quantization block (or per element for F32 tensors),
// writing GGUF-order bytes.
__global__ void synth_kernel(uint8_t *dst, int type, uint64_t nunits, uint64_t key, int kind) {
    for (uint64_t b = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; b < nunits;
         b += uint64_t(gridDim.x) * blockDim.x) {
        if (type == QMA_TYPE_F32) {
            reinterpret_cast<float *>(dst)[b] = kind_value(kind, key, b);
            continue;
        }
        float v[256];
        const int per = type == QMA_TYPE_Q8_0 ? 32 : 256;
        for (int i = 0; i < per; i++) v[i] = kind_value(kind, key, b * per + i);
        if (type == QMA_TYPE_Q4_K) quantize_q4k(v, dst + b * Q4K_BYTES);
        else if (type == QMA_TYPE_Q6_K) quantize_q6k(v, dst + b * Q6K_BYTES);
        else quantize_q80(v, dst + b * Q80_BYTES);
    }
}

int synth_tensor_gguf(const char *name, int type, uint64_t nelem, uint64_t seed, void *dst,
                      cudaStream_t st) {
    const uint64_t per = type == QMA_TYPE_F32 ? 1 : (type == QMA_TYPE_Q8_0 ? 32 : 256);
    const uint64_t nunits = nelem / per;
    const uint64_t key = name_key(name, seed);
    const int kind = tensor_kind(name);
    const int threads = 128;
    uint64_t blocks = (nunits + threads - 1) / threads;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks == 0) blocks = 1;
    synth_kernel<<<unsigned(blocks), threads, 0, st>>>(static_cast<uint8_t *>(dst), type, nunits,
                                                       key, kind);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

}  // namespace qma

extern "C" int qma_cuda_synth_tensor(const char *name, int type, uint64_t nelem, uint64_t seed,
                                     void *dst, void *stream) {
    qma::clear_error();
    QMA_REQUIRE(name && dst && nelem > 0, "qma_cuda_synth_tensor: bad arguments");
    QMA_REQUIRE(type == QMA_TYPE_F32 || type == QMA_TYPE_Q4_K || type == QMA_TYPE_Q6_K ||
                    type == QMA_TYPE_Q8_0,
                "qma_cuda_synth_tensor: unsupported type %d", type);
    QMA_REQUIRE(type == QMA_TYPE_F32 || nelem % (type == QMA_TYPE_Q8_0 ? 32 : 256) == 0,
                "qma_cuda_synth_tensor: %llu elements is not a whole number of blocks",
                (unsigned long long)nelem);
    return qma::synth_tensor_gguf(name, type, nelem, seed, dst, qma::as_stream(stream));
}
