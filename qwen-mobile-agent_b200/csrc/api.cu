// api.cu -- library-level entry points: error reporting, device selection,
// packed weight layouts (qma_cuda.h).
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace qma {

static thread_local char g_err[512];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

bool pdl_enabled() { return true; }

#ifdef QMA_TRACE
__device__ unsigned long long g_trace[TRACE_CAP][2];
__device__ unsigned g_trace_n;
#endif

size_t packed_bytes(int wtype, int rows, int n) {
    switch (wtype) {
    case QMA_TYPE_Q4_K: return size_t(rows) * (n / QK) * Q4K_BYTES;
    case QMA_TYPE_Q6_K:
        return pad16(q6_plane_ql(rows, n)) + pad16(q6_plane_qh(rows, n)) +
               pad16(q6_plane_sc(rows, n)) + pad16(q6_plane_d(rows, n));
    case QMA_TYPE_Q8_0: return pad16(size_t(rows) * n) + pad16(size_t(rows) * (n / 32) * 2);
    case QMA_TYPE_F32: return size_t(rows) * n * 4;
    default: return 0;
    }
}

// GGUF Q6_K block (ql[128] qh[64] scales[16] d) -> planes, ql/qh chunks
// swizzled (q6_ql_chunk / q6_qh_chunk); one thread per block.
__global__ void repack_q6k_kernel(const uint8_t *__restrict__ src, int rows, int n,
                                  uint8_t *ql, uint8_t *qh, int8_t *sc, __half *d) {
    const int nb = n / QK;
    const long total = long(rows) * nb;
    for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total;
         i += long(gridDim.x) * blockDim.x) {
        const long r = i / nb, b = i % nb;
        const uint8_t *s = src + i * Q6K_BYTES;
        uint8_t *oql = ql + r * (n / 2) + b * 128;
        uint8_t *oqh = qh + r * (n / 4) + b * 64;
        int8_t *osc = sc + r * (n / 16) + b * 16;
        const int seg = int(i & 0x7fffffff);   // only s mod 4 matters
        for (int k = 0; k < 128; k++) oql[(q6_ql_chunk(k >> 4, seg) << 4) | (k & 15)] = s[k];
        for (int k = 0; k < 64; k++) oqh[(q6_qh_chunk(k >> 4, seg) << 4) | (k & 15)] = s[128 + k];
        for (int k = 0; k < 16; k++) osc[k] = static_cast<int8_t>(s[192 + k]);
        d[r * nb + b] = __ushort_as_half(uint16_t(s[208] | (s[209] << 8)));
    }
}

// GGUF Q8_0 block (d, q[32]) -> planes; one thread/block.
__global__ void repack_q80_kernel(const uint8_t *__restrict__ src, int rows, int n, int8_t *q,
                                  __half *d) {
    const int nb = n / 32;
    const long total = long(rows) * nb;
    for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total;
         i += long(gridDim.x) * blockDim.x) {
        const uint8_t *s = src + i * Q80_BYTES;
        d[i] = __ushort_as_half(uint16_t(s[0] | (s[1] << 8)));
        int8_t *o = q + i * 32;
        for (int k = 0; k < 32; k++) o[k] = static_cast<int8_t>(s[2 + k]);
    }
}

int repack(int wtype, const void *src, int rows, int n, void *dst, cudaStream_t st) {
    const uint8_t *s = static_cast<const uint8_t *>(src);
    uint8_t *o = static_cast<uint8_t *>(dst);
    if (wtype == QMA_TYPE_Q4_K || wtype == QMA_TYPE_F32) {
        QMA_CHECK_CUDA(cudaMemcpyAsync(dst, src, packed_bytes(wtype, rows, n),
                                       cudaMemcpyDeviceToDevice, st));
        return QMA_CUDA_OK;
    }
    if (wtype == QMA_TYPE_Q6_K) {
        uint8_t *ql = o;
        uint8_t *qh = ql + pad16(q6_plane_ql(rows, n));
        int8_t *sc = reinterpret_cast<int8_t *>(qh + pad16(q6_plane_qh(rows, n)));
        __half *d = reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(sc) +
                                               pad16(q6_plane_sc(rows, n)));
        const long nblk = long(rows) * (n / QK);
        const int grid = int((nblk + 255) / 256 < 65535 ? (nblk + 255) / 256 : 65535);
        repack_q6k_kernel<<<grid, 256, 0, st>>>(s, rows, n, ql, qh, sc, d);
        QMA_CHECK_LAUNCH();
        return QMA_CUDA_OK;
    }
    if (wtype == QMA_TYPE_Q8_0) {
        int8_t *q = reinterpret_cast<int8_t *>(o);
        __half *d = reinterpret_cast<__half *>(o + pad16(size_t(rows) * n));
        const long nblk = long(rows) * (n / 32);
        const int grid = int((nblk + 255) / 256 < 65535 ? (nblk + 255) / 256 : 65535);
        repack_q80_kernel<<<grid, 256, 0, st>>>(s, rows, n, q, d);
        QMA_CHECK_LAUNCH();
        return QMA_CUDA_OK;
    }
    set_error("repack: unsupported weight type %d", wtype);
    return QMA_CUDA_ERR_UNSUPPORTED;
}

}  // namespace qma

extern "C" {

int qma_cuda_abi_version(void) { return QMA_CUDA_ABI_VERSION; }

const char *qma_cuda_last_error(void) { return qma::g_err; }

int qma_cuda_init(int device) {
    qma::clear_error();
    int n = 0;
    QMA_CHECK_CUDA(cudaGetDeviceCount(&n));
    QMA_REQUIRE(device >= 0 && device < n, "qma_cuda_init: device %d of %d", device, n);
    QMA_CHECK_CUDA(cudaSetDevice(device));
    cudaDeviceProp p;
    QMA_CHECK_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10) {
        qma::set_error("qma_cuda_init: device %d is sm_%d%d, this build targets sm_100a", device,
                       p.major, p.minor);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    return QMA_CUDA_OK;
}

size_t qma_cuda_packed_bytes(int wtype, int rows, int n) { return qma::packed_bytes(wtype, rows, n); }

int qma_cuda_repack(int wtype, const void *src, int rows, int n, void *dst, void *stream) {
    qma::clear_error();
    QMA_REQUIRE(src && dst && rows > 0 && n > 0 && n % 256 == 0, "qma_cuda_repack: bad arguments");
    return qma::repack(wtype, src, rows, n, dst, qma::as_stream(stream));
}

}  // extern "C"

#ifdef QMA_TRACE
// Trace build only: copy up to `cap` records (2 x u64 each) to `out`, return
// how many were written since the last reset, and reset the ring.
extern "C" int qma_trace_read(unsigned long long *out, int cap) {
    unsigned n = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    cudaMemcpyFromSymbol(&n, qma::g_trace_n, sizeof(n));
    const unsigned k = n < unsigned(cap) ? n : unsigned(cap);
    if (k) cudaMemcpyFromSymbol(out, qma::g_trace, size_t(k) * 16);
    const unsigned zero = 0;
    cudaMemcpyToSymbol(qma::g_trace_n, &zero, sizeof(zero));
    return int(n);
}
#endif
