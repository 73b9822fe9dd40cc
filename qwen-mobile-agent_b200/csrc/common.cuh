// common.cuh -- shared device/host helpers of the qma B200 engine (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>

#include "qma_cuda.h"

namespace qma {

// ------------------------------------------------------------ error plumbing
// Thread-local message behind qma_cuda_last_error(); every C entry point
// returns a status and never exits the process.
void set_error(const char *fmt, ...);
void clear_error();

#define QMA_CHECK_CUDA(call)                                                   \
    do {                                                                       \
        cudaError_t e_ = (call);                                               \
        if (e_ != cudaSuccess) {                                               \
            ::qma::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call,        \
                             cudaGetErrorString(e_));                          \
            return QMA_CUDA_ERR_CUDA;                                          \
        }                                                                      \
    } while (0)

#define QMA_CHECK_LAUNCH()                                                     \
    do {                                                                       \
        cudaError_t e_ = cudaGetLastError();                                   \
        if (e_ != cudaSuccess) {                                               \
            ::qma::set_error("%s:%d kernel launch: %s", __FILE__, __LINE__,    \
                             cudaGetErrorString(e_));                          \
            return QMA_CUDA_ERR_CUDA;                                          \
        }                                                                      \
    } while (0)

#define QMA_REQUIRE(cond, ...)                                                 \
    do {                                                                       \
        if (!(cond)) {                                                         \
            ::qma::set_error(__VA_ARGS__);                                     \
            return QMA_CUDA_ERR_INVALID;                                       \
        }                                                                      \
    } while (0)

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
// Device buffers handed across the C ABI are read with 16-byte vector loads.
static inline bool aligned_to(const void *p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

// ------------------------------------------------------------ block formats
constexpr int QK = 256;            // super-block lanes (QK_K, qma.h:74)
constexpr int Q4K_BYTES = 144;     // block_q4_K, qma.h:77-82
constexpr int Q6K_BYTES = 210;     // block_q6_K, qma.h:85-90
constexpr int Q80_BYTES = 34;      // block_q8_0, qma.h:92-94

// Packed (planar) layouts of Q6_K and Q8_0 matrices; see qma_cuda.h.
struct Q6Planes {
    const uint8_t *ql, *qh;
    const int8_t *sc;
    const __half *d;
};
struct Q8Planes {
    const int8_t *q;
    const __half *d;
};
__host__ __device__ inline size_t pad16(size_t x) { return (x + 15) & ~size_t(15); }
__host__ __device__ inline size_t q6_plane_ql(int rows, int n) { return size_t(rows) * n / 2; }
__host__ __device__ inline size_t q6_plane_qh(int rows, int n) { return size_t(rows) * n / 4; }
__host__ __device__ inline size_t q6_plane_sc(int rows, int n) { return size_t(rows) * n / 16; }
__host__ __device__ inline size_t q6_plane_d(int rows, int n) { return size_t(rows) * (n / 256) * 2; }

// Q6_K plane swizzle.  A segment is one (row, super-block) of a plane:
// 128 B of ql (8 chunks of 16 B), 64 B of qh (4 chunks); s = row * (n/256)
// + sb numbers the segments.  Chunk c of a ql segment is stored at chunk
// c ^ (s & 3), chunk c of a qh segment at c ^ ((s >> 1) & 1).  The 8 lanes of
// a quarter warp that read the same chunk of their unit from 4 consecutive
// segments then hit 8 different 16-byte bank groups of shared memory (a
// plain layout puts them on 2).  The key depends on s mod 4 only, so a copy
// of rows r0.. with r0 * (n/256) a multiple of 4 keeps it.
__host__ __device__ inline int q6_ql_chunk(int c, int s) { return c ^ (s & 3); }
__host__ __device__ inline int q6_qh_chunk(int c, int s) { return c ^ ((s >> 1) & 1); }

__host__ __device__ inline Q6Planes q6_planes(const void *base, int rows, int n) {
    const uint8_t *p = static_cast<const uint8_t *>(base);
    Q6Planes P;
    P.ql = p;
    p += pad16(q6_plane_ql(rows, n));
    P.qh = p;
    p += pad16(q6_plane_qh(rows, n));
    P.sc = reinterpret_cast<const int8_t *>(p);
    p += pad16(q6_plane_sc(rows, n));
    P.d = reinterpret_cast<const __half *>(p);
    return P;
}
inline Q8Planes q8_planes(const void *base, int rows, int n) {
    const uint8_t *p = static_cast<const uint8_t *>(base);
    Q8Planes P;
    P.q = reinterpret_cast<const int8_t *>(p);
    P.d = reinterpret_cast<const __half *>(p + pad16(size_t(rows) * n));
    return P;
}
size_t packed_bytes(int wtype, int rows, int n);
// GGUF-order device matrix -> packed layout (api.cu)
int repack(int wtype, const void *src, int rows, int n, void *dst, cudaStream_t st);

// ------------------------------------------------------------ device helpers
// Streaming 16-byte load of weights: read once per step, keep out of L1.
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_stream8(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(v.x), "=r"(v.y)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_stream4(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ld_stream2(const void *p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Eight warp-wide sums at once (9 shuffles): afterwards lane l holds the sum
// over the warp of v[warp_sum8_index(l)].
__device__ __forceinline__ int warp_sum8_index(int lane) {
    return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}
__device__ __forceinline__ float warp_sum8(const float (&v)[8], int lane) {
    float a[4];
    const bool h16 = lane & 16;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float mine = h16 ? v[4 + i] : v[i], other = h16 ? v[i] : v[4 + i];
        a[i] = mine + __shfl_xor_sync(0xffffffffu, other, 16);
    }
    float b[2];
    const bool h8 = lane & 8;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float mine = h8 ? a[2 + i] : a[i], other = h8 ? a[i] : a[2 + i];
        b[i] = mine + __shfl_xor_sync(0xffffffffu, other, 8);
    }
    const bool h4 = lane & 4;
    float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}
// Four warp-wide sums at once (6 shuffles): afterwards lane l holds the sum
// over the warp of v[warp_sum4_index(l)].
__device__ __forceinline__ int warp_sum4_index(int lane) { return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1); }
__device__ __forceinline__ float warp_sum4(const float (&v)[4], int lane) {
    float a[2];
    const bool h16 = lane & 16;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float mine = h16 ? v[2 + i] : v[i], other = h16 ? v[i] : v[2 + i];
        a[i] = mine + __shfl_xor_sync(0xffffffffu, other, 16);
    }
    const bool h8 = lane & 8;
    float c = (h8 ? a[1] : a[0]) + __shfl_xor_sync(0xffffffffu, h8 ? a[0] : a[1], 8);
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}
// Sum over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int width) {
    for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int group_sum_i(int v, int width) {
    for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Programmatic dependent launch: wait for the upstream grid's writes, and
// let the downstream grid start its prologue.  No-ops without PDL.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// Asynchronous L2 prefetch of a byte range (16-byte aligned address, size a
// multiple of 16): weights are requested before the data they combine with
// is ready.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// Any byte range: shrunk to the 16-byte-aligned range inside it, so it never
// reaches outside [p, p + bytes) (the allocation holding it starts 256-byte
// aligned, so rounding the start down stays inside it as well).
__device__ __forceinline__ void prefetch_l2_range(const void *p, size_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p) & ~uintptr_t(15);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
    for (uintptr_t q = a; q < e; q += (uintptr_t(1) << 30)) {
        const uintptr_t n = e - q < (uintptr_t(1) << 30) ? e - q : (uintptr_t(1) << 30);
        prefetch_l2(reinterpret_cast<const void *>(q), uint32_t(n));
    }
}

// ------------------------------------------- bulk copies into shared memory --
// Global -> this CTA's shared memory through the TMA engine (non-tensor
// cp.async.bulk into this CTA alone), completion counted in bytes on an mbarrier.
// Addresses 16-byte aligned, sizes multiples of 16.
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// A large range as many 4 KB bulk copies issued by the 32 lanes of a warp
// (the mbarrier's byte count must already be armed): the TMA engine keeps
// several copies in flight, a single large one streams slowly.
constexpr uint32_t BULK_PIECE = 4096;
__device__ __forceinline__ void bulk_g2s_warp(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              int lane) {
    uint8_t *d = static_cast<uint8_t *>(dst);
    const uint8_t *s = static_cast<const uint8_t *>(src);
    for (uint32_t off = uint32_t(lane) * BULK_PIECE; off < bytes; off += 32 * BULK_PIECE)
        bulk_g2s(d + off, s + off, bytes - off < BULK_PIECE ? bytes - off : BULK_PIECE, bar);
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier: false after `limit` polls
// (each poll may suspend the thread for a hardware-defined time).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = 1u << 22) {
    for (uint32_t i = 0; i < limit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Thread-block cluster helpers (split arrive / wait of the cluster barrier,
// and a load from another CTA's shared memory).
__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
    cluster_arrive();
    cluster_wait();
}
// address of `p` (this CTA's shared memory) in the shared memory of CTA `rank`
template <class T> __device__ __forceinline__ T *cluster_map(T *p, unsigned rank) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p)), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return reinterpret_cast<T *>(static_cast<uintptr_t>(r));
}
__device__ __forceinline__ float ld_cluster_f32(const float *remote) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];"
                 : "=f"(v)
                 : "r"(static_cast<uint32_t>(reinterpret_cast<uintptr_t>(remote)))
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_cluster_f64(double *remote, double v) {
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(static_cast<uint32_t>(reinterpret_cast<uintptr_t>(remote))),
                 "d"(v)
                 : "memory");
}
__device__ __forceinline__ void st_cluster_f32(float *remote, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(static_cast<uint32_t>(reinterpret_cast<uintptr_t>(remote))),
                 "f"(v)
                 : "memory");
}

// Kernel launch with optional thread-block cluster and programmatic
// dependent launch (the kernel may start while the previous kernel on the
// stream finishes; it must call pdl_wait() before touching that kernel's
// outputs or writing anything it reads).
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_ex(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, int cluster, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    unsigned n = 0;
    if (cluster > 1) {
        at[n].id = cudaLaunchAttributeClusterDimension;
        at[n].val.clusterDim.x = unsigned(cluster);
        at[n].val.clusterDim.y = 1;
        at[n].val.clusterDim.z = 1;
        n++;
    }
    if (pdl) {
        at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    cfg.attrs = at;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Programmatic dependent launch of the engine's kernels (on by default).
bool pdl_enabled();

// One-time set-up that CUDA keeps per device (kernel attributes such as the
// dynamic shared-memory limit or non-portable cluster sizes): one bit per
// device that has it.  A process that drives several GPUs sets it on each
// device at that device's first call.  Devices past 63 redo it every call.
struct PerDevice {
    std::atomic<unsigned long long> mask{0};
    static int current() {
        int d = 0;
        if (cudaGetDevice(&d) != cudaSuccess) d = 0;
        return d;
    }
    bool done() const {
        const int d = current();
        return d < 64 && ((mask.load(std::memory_order_acquire) >> d) & 1ull);
    }
    void mark() {
        const int d = current();
        if (d < 64) mask.fetch_or(1ull << d, std::memory_order_acq_rel);
    }
};

// Byte ranges (weights) the first kernel of a layer asks L2 to fetch ahead
// of the kernels that use them.
struct Prefetch {
    static constexpr int N = 6;
    const void *p[N] = {};
    size_t bytes[N] = {};
};

// ---------------------------------------------------------------- tracing --
// Built with -DQMA_TRACE, every CTA of the forward kernels appends
// {kernel id, CTA, entry ns, exit ns} (the GPU's global timer) to a device
// ring, read back with qma_trace_read(); otherwise QMA_TRACE_SCOPE is empty.
enum TraceKernel : uint32_t {
    TK_EMBED = 1, TK_RMSNORM, TK_GEMV, TK_CONV, TK_GDN, TK_GATED_NORM, TK_QK_PREP, TK_ATTN_CHUNK,
    TK_ATTN_COMBINE, TK_SALIENCE, TK_ROUTER, TK_EXPERT, TK_ARGMAX, TK_MOE_NORM
};
#ifdef QMA_TRACE
constexpr uint32_t TRACE_CAP = 1u << 22;
extern __device__ unsigned long long g_trace[TRACE_CAP][2];
extern __device__ unsigned g_trace_n;
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long v;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(v));
    return v;
}
struct TraceScope {
    uint32_t id;
    unsigned long long t0;
    __device__ explicit TraceScope(uint32_t k) : id(k), t0(threadIdx.x == 0 ? gtimer() : 0) {}
    __device__ ~TraceScope() {
        if (threadIdx.x == 0) {
            const unsigned i = atomicAdd(&g_trace_n, 1u) % TRACE_CAP;
            const unsigned cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
            g_trace[i][0] = (static_cast<unsigned long long>(id) << 56) |
                            (static_cast<unsigned long long>(cta & 0xffffff) << 32) | (t0 & 0xffffffffull);
            g_trace[i][1] = gtimer();
        }
    }
};
#define QMA_TRACE_SCOPE(k) ::qma::TraceScope qma_trace_scope_(k)
// a point event `phase` of kernel k, recorded by thread 0 of the first CTA
__device__ __forceinline__ void trace_mark(uint32_t k, uint32_t phase) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) {
        const unsigned i = atomicAdd(&g_trace_n, 1u) % TRACE_CAP;
        const unsigned long long t = gtimer();
        g_trace[i][0] = (static_cast<unsigned long long>(k | 0x80u) << 56) |
                        (static_cast<unsigned long long>(phase) << 32) | (t & 0xffffffffull);
        g_trace[i][1] = t;
    }
}
#define QMA_TRACE_MARK(k, phase) ::qma::trace_mark(k, phase)
#else
#define QMA_TRACE_SCOPE(k) do {} while (0)
#define QMA_TRACE_MARK(k, phase) do {} while (0)
#endif

// The fp32 fold of one super-block's exact integer sums into a grouped
// GEMM accumulator, in one fixed operation order (explicit roundings, no
// contraction), shared by the tensor-core GEMM kernels of both generations so
// that they produce the same bits: Q4_K adds xd * (d * I1 - dmin * I2)
// (dot_q4_K_q8k, q8k.c:89-131), Q6_K adds d * xd * I (dot_q6_K_q8k,
// q8k.c:210-262).
__device__ __forceinline__ float q4k_fold(float acc, float xd, float d, float dmin, int I1, int I2) {
    return __fadd_rn(acc, __fmul_rn(xd, __fsub_rn(__fmul_rn(d, float(I1)), __fmul_rn(dmin, float(I2)))));
}
__device__ __forceinline__ float q6k_fold(float acc, float xd, float d, int I) {
    return __fadd_rn(acc, __fmul_rn(__fmul_rn(d, xd), float(I)));
}

// I2 = sum_j m_j (s_2j + s_2j+1) of one Q4_K super-block: the eight 6-bit
// mins m_j against the Q8_K activation's sixteen 16-lane sums s (int16 at p,
// 16-byte aligned), as eight 2-way 16 x 8-bit integer dot products over
// byte-duplicated mins (md[i] = bytes m_2i, m_2i, m_2i+1, m_2i+1).  Exact:
// the same integer as the plain sum.
__device__ __forceinline__ void q4k_mins_dup(const int (&mn)[8], int (&md)[4]) {
#pragma unroll
    for (int i = 0; i < 4; i++) md[i] = (mn[2 * i] * 0x0101) | ((mn[2 * i + 1] * 0x0101) << 16);
}
__device__ __forceinline__ int q4k_i2(const int16_t *p, const int (&md)[4]) {
    const int4 u = __ldg(reinterpret_cast<const int4 *>(p)), v = __ldg(reinterpret_cast<const int4 *>(p) + 1);
    int r = __dp2a_lo(u.x, md[0], 0);
    r = __dp2a_hi(u.y, md[0], r);
    r = __dp2a_lo(u.z, md[1], r);
    r = __dp2a_hi(u.w, md[1], r);
    r = __dp2a_lo(v.x, md[2], r);
    r = __dp2a_hi(v.y, md[2], r);
    r = __dp2a_lo(v.z, md[3], r);
    return __dp2a_hi(v.w, md[3], r);
}

// 6-bit scale/min unpack of a Q4_K super-block (get_scale_min_k4,
// quants.c:18-26 / q8k.c:22-30).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *s, int &d, int &m) {
    if (j < 4) {
        d = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        d = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

}  // namespace qma
