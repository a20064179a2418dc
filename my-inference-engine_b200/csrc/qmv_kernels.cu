// sm_100a kernels for the GGUF quantized matrix-vector path.
//
//  * repack      raw GGUF blocks -> chunk-major resident rows (once per upload).
//  * dequant     bit-exact block decoding (same float bits as the reference's
//                *_dequantize_block, src/quantization.cpp:54-67, 161-184,
//                380-409, 588-615, including x86 NaN payload rules).
//  * gemv        y = W x with in-register dequantisation and dp4a integer dots.
//  * matmul      Y = W X for a batch of positions; each weight chunk is loaded
//                once and applied to every position
//                (src/quantized_matvec.cpp:164-224).
//  * argmax      greedy selection fused into the gemv epilogue, or standalone
//                (src/sampler.cpp:14-36).
//
// Integer inner loop.  Each 32-element block of x is quantized on the fly
// into 16-bit integers xq = rint(x / s) held as two int8 planes
// (hi = (xq + 128) >> 8, lo = xq - 256 hi), where s is the power of two that
// puts max|xq| in (16320, 32639].  A block dot is then
// s * (256 * dp4a(w, hi) + dp4a(w, lo)) with exact 32-bit integer sums; the
// quantisation error of x is at most 2^-15 of the block maximum (zero for
// dyadic inputs), far inside the parity bound |y - y_ref| <= 1e-4 * sum|w x|.
// Blocks whose maximum is below 2^-100 share the scale 2^-114, so magnitudes
// under 2^-115 quantize to zero.  The Q5_0 (-16) and Q6_K (-32) offsets and
// the Q4_K minimum use per-16-element sums of xq.
//
// Shared-memory x layout mirrors the weight layout: the 16-element slice j
// of chunk c is stored at (j * C + c) * 16 in each plane, with one record
// {s, s * sum of xq} per slice, so lanes reading consecutive chunks hit
// consecutive banks.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "qmv_internal.h"

namespace qmv {

namespace {

constexpr int kThreads = 256;
constexpr unsigned kFull = 0xffffffffu;

__host__ __device__ constexpr uint32_t pad16(uint32_t v) { return (v + 15u) & ~15u; }

// ---------------------------------------------------------------- helpers

// IEEE binary16 -> binary32 from the bit pattern, exact for every encoding,
// with the reference's NaN quieting (src/quantization.cpp:23-49).
__device__ __forceinline__ float f16_exact(uint32_t h)
{
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0u) {
        if (m == 0u) {
            bits = sign;
        } else {
            int sh = __clz(m) - 21;  // moves the leading one to bit 10
            bits = sign | ((uint32_t)(113 - sh) << 23) | (((m << sh) & 0x3ffu) << 13);
        }
    } else if (e == 31u) {
        bits = sign | 0x7f800000u | (m << 13) | (m ? 0x00400000u : 0u);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

// Hardware fp16 conversion for the dot-product path (identical to f16_exact
// for every non-NaN encoding).
__device__ __forceinline__ float f16_fast(uint32_t h)
{
    return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

// Streaming 128-bit load of packed weights: read-only, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const uint8_t *p)
{
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_stream32(const uint8_t *p)
{
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_stream16(const uint8_t *p)
{
    unsigned short v;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c)
{
    return __dp4a((int)a, (int)b, c);
}

// Argmax key: high word orders the value (after folding -0 into +0), low word
// is 0xFFFFFFFF - index so that ties keep the lowest index
// (src/sampler.cpp:29-31).  NaN/Inf -> all ones.
__device__ __forceinline__ unsigned long long make_key(float v, int index)
{
    uint32_t u = __float_as_uint(v);
    if ((u & 0x7f800000u) == 0x7f800000u) return ~0ull;
    if ((u & 0x7fffffffu) == 0u) u = 0u;
    uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)index);
}

__device__ __forceinline__ unsigned long long max_ull(unsigned long long a, unsigned long long b)
{
    return a > b ? a : b;
}

// CTA-wide max of one key per thread; result valid in thread 0.
__device__ unsigned long long block_max_key(unsigned long long k, unsigned long long *scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k = max_ull(k, __shfl_xor_sync(kFull, k, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = k;
    __syncthreads();
    if (warp == 0) {
        k = lane < (int)(blockDim.x >> 5) ? scratch[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) k = max_ull(k, __shfl_xor_sync(kFull, k, o));
    }
    return k;
}

// Fold this CTA's key (valid in thread 0) into the workspace's running
// maximum (an atomic max, then an arrival counted with release semantics);
// the last CTA to arrive (acquire) copies the maximum to *am.key and re-arms
// the slot and the counter.  No CTA waits on another, and no CTA but the last
// reads anything back beyond its own arrival.  Workspace: u32 counter at 0,
// u64 running maximum at 8 (both zero between launches).
__device__ void finish_argmax(unsigned long long cta_key, const ArgmaxOut &am, unsigned long long *scratch)
{
    (void)scratch;
    if (threadIdx.x != 0) return;
    unsigned int *counter = reinterpret_cast<unsigned int *>(am.workspace);
    unsigned long long *slot =
        reinterpret_cast<unsigned long long *>(reinterpret_cast<uint8_t *>(am.workspace) + 8);
    atomicMax(slot, cta_key);
    unsigned int prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
    if (prev != gridDim.x - 1u) return;
    unsigned long long k;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(k) : "l"(slot) : "memory");
    *am.key = k;
    *slot = 0ull;
    *counter = 0u;
}

// ------------------------------------------------------ peer exchange
//
// Row-sharded projection across the GPUs of one node.  Every CTA copies the
// logits of its own contiguous rows into each peer's slot for this rank
// (coalesced NVLink stores), writes its argmax key into every rank's key
// table, fences at system scope and release-stores the epoch into its own
// flag in every rank's buffer (plain stores and loads over NVLink, no remote
// atomics).  No CTA waits for the others of its rank before signalling.  The
// rank's last CTA to finish (a local counter) waits until every source CTA's
// flag of every rank shows this epoch, folds the world * ncta keys and
// advances the epoch.  After the kernel every rank holds all logits and the
// same global key.

__device__ unsigned int g_peer_status;

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p)
{
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// This launch's epoch (the counter is only stored back by the last CTA after
// every CTA has read it).
__device__ __forceinline__ unsigned int exchange_epoch(const Exchange &ex)
{
    return *((volatile unsigned int *)ex.epoch) + 1u;
}

// This CTA's part of the exchange (all threads): its rows [r0, r1) of this
// rank's slot to every peer, its key into every rank's table, then the
// release of its flag.  cta_key is valid in thread 0.
__device__ void exchange_send(const Exchange &ex, int par, unsigned int epoch, const float *y_local, int r0, int r1,
                              unsigned long long cta_key)
{
    for (int p = 0; p < ex.world; ++p) {
        if (p == ex.rank) continue;
        float *dst = ex.logits[par][p] + (size_t)ex.rank * ex.slot_rows;
        for (int i = r0 + (int)threadIdx.x; i < r1; i += blockDim.x) dst[i] = y_local[i];
    }
    if (threadIdx.x == 0)
        for (int p = 0; p < ex.world; ++p) ex.keys[par][p][ex.rank * kMaxExCtas + blockIdx.x] = cta_key;
    // The barrier orders every thread's peer stores before thread 0's
    // system-scope fence and the release of the flags.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < ex.world; ++p) st_release_sys(ex.flags[par][p] + ex.rank * kMaxExCtas + blockIdx.x, epoch);
    }
}

// The rank's last CTA: wait (bounded) for every rank's CTAs of this epoch,
// fold all keys, advance the epoch.  A CTA whose flag never arrives leaves
// key 0 (no token) and sets g_peer_status.
__device__ void exchange_collect(const Exchange &ex, int par, unsigned int epoch, unsigned long long *out_key,
                                 unsigned long long *scratch)
{
    __shared__ int ok;
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    const unsigned int *flags = ex.flags[par][ex.rank];
    const unsigned long long t0 = globaltimer_ns();
    for (int e = threadIdx.x; e < ex.world * ex.ncta; e += blockDim.x) {
        const unsigned int *f = flags + (e / ex.ncta) * kMaxExCtas + e % ex.ncta;
        for (uint32_t n = 1; ld_acquire_sys(f) != epoch; ++n) {
            if ((n & 63u) == 0u && globaltimer_ns() - t0 > 2000000000ull) {
                atomicOr(&g_peer_status, 1u);
                ok = 0;
                break;
            }
        }
        if (!*(volatile int *)&ok) break;
    }
    __syncthreads();
    unsigned long long k = 0ull;
    if (ok) {
        const unsigned long long *keys = ex.keys[par][ex.rank];
        for (int e = threadIdx.x; e < ex.world * ex.ncta; e += blockDim.x)
            k = max_ull(k, __ldcg(keys + (e / ex.ncta) * kMaxExCtas + e % ex.ncta));
    }
    k = block_max_key(k, scratch);
    if (threadIdx.x == 0) {
        *out_key = ok ? k : 0ull;  // 0 decodes as "no token"
        *ex.epoch = epoch;
    }
}

// ------------------------------------------------------- x quantisation

// Slices of 16 x values per chunk and the chunk-major index of the slice
// that starts at position p (a multiple of 16).
template <uint32_t FMT> struct Slices;
template <> struct Slices<kQ8_0> {
    static __device__ __forceinline__ int index(int p, int C) { return ((p >> 4) & 1) * C + (p >> 5); }
};
template <> struct Slices<kQ5_0> {
    static __device__ __forceinline__ int index(int p, int C) { return ((p >> 4) & 1) * C + (p >> 5); }
};
template <> struct Slices<kQ4_K> {
    static __device__ __forceinline__ int index(int p, int C) { return ((p >> 4) & 3) * C + (p >> 6); }
};
template <> struct Slices<kQ6_K> {
    static __device__ __forceinline__ int index(int p, int C)
    {
        return ((p >> 5) & 3) * C + 2 * (p >> 7) + ((p >> 4) & 1);
    }
};

// Quantized x of one position in shared memory.
struct XS {
    const uint8_t *hi;   // [cols] int8, chunk-major slices
    const uint8_t *lo;   // [cols]
    const float2 *rec;   // [cols/16] {s, s * sum of xq}; s is NaN for a non-finite block
    __device__ __forceinline__ uint4 h(int j, int C, int c) const
    {
        return *reinterpret_cast<const uint4 *>(hi + ((j * C + c) << 4));
    }
    __device__ __forceinline__ uint4 l(int j, int C, int c) const
    {
        return *reinterpret_cast<const uint4 *>(lo + ((j * C + c) << 4));
    }
    __device__ __forceinline__ float2 r(int j, int C, int c) const { return rec[j * C + c]; }
};

// Bytes of one quantized position, rounded up to 16 so consecutive positions
// keep the 16-byte alignment of their 128-bit shared loads.
__host__ __device__ constexpr size_t xs_bytes(int cols)
{
    return (2 * (size_t)cols + (size_t)cols / 2 + 15) & ~(size_t)15;
}

__device__ __forceinline__ XS xs_view(const uint8_t *base, int cols)
{
    XS s;
    s.hi = base;
    s.lo = base + cols;
    s.rec = reinterpret_cast<const float2 *>(base + 2 * cols);
    return s;
}

// Quantize x[0..cols) into shared memory (every thread of the CTA takes part;
// 8 consecutive lanes own one 32-element block, 4 lanes one 16-element slice).
// np > 1 quantizes the rows x[p * cols ..] of np positions in one pass (the
// float4s of all positions form one contiguous range, and a 32-element block
// never straddles two positions since cols is a multiple of 32), so the
// global-load latency is paid once; position p goes to base + p * pos_bytes.
// pre (kPreRmsNorm / kPreSwiGlu, one position): the x of a fused prologue,
// formed element-wise as it is loaded (denom = sqrt(mean(x^2) + eps)).
// special (shared, optional): set to 1 when a block holds a NaN/Inf or is
// nonzero with every magnitude below 2^-100 (the blocks the integer path would
// turn into NaN or flush); the kernel then computes its rows in fp32.
// LIVE: x and aux were written earlier in the same launch (the persistent
// decode step), so they are read through L2 rather than the read-only path.
// ss (kPreScale): this thread's sum of x^2 is added to *ss.
template <uint32_t FMT, int NT = kThreads, bool LIVE = false>
__device__ void quantize_x(const float *__restrict__ x, int cols, int C, uint8_t *base, int np = 1,
                           size_t pos_bytes = 0, int pre = kPreNone, float denom = 1.f,
                           const float *__restrict__ aux = nullptr, int *special = nullptr, float *ss = nullptr)
{
    const int n4 = cols >> 2;
    const int total = np * n4;
    constexpr int U = 8;
    for (int it0 = 0; it0 * NT < total; it0 += U) {
        // every load of the batch is issued at once (predicated past the
        // end); the prologue arithmetic then runs only for the valid part
        float4 v[U], w4[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int g = (it0 + u) * NT + threadIdx.x;
            v[u] = g >= total ? make_float4(0.f, 0.f, 0.f, 0.f)
                   : LIVE     ? __ldcg(reinterpret_cast<const float4 *>(x) + g)
                              : __ldg(reinterpret_cast<const float4 *>(x) + g);
            if (pre != kPreNone)
                w4[u] = g >= total ? make_float4(0.f, 0.f, 0.f, 0.f)
                        : LIVE     ? __ldcg(reinterpret_cast<const float4 *>(aux) + g)
                                   : __ldg(reinterpret_cast<const float4 *>(aux) + g);
        }
        if (pre != kPreNone) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if ((it0 + u) * NT >= total) break;  // uniform across the CTA
                const int g = (it0 + u) * NT + threadIdx.x;
                if (g >= total) continue;
                const float4 b = w4[u];
                if (pre == kPreRmsNorm) {
                    v[u] = make_float4((v[u].x / denom) * b.x, (v[u].y / denom) * b.y, (v[u].z / denom) * b.z,
                                       (v[u].w / denom) * b.w);
                } else if (pre == kPreScale) {
                    *ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
                    v[u] = make_float4(v[u].x * b.x, v[u].y * b.y, v[u].z * b.z, v[u].w * b.w);
                } else {
                    // SwiGLU: the x that is quantized next (to 2^-15 of its
                    // block maximum), so the fast exponential's few-ulp error
                    // is far below what the quantization keeps
                    v[u] = make_float4(b.x * (v[u].x / (1.f + __expf(-v[u].x))),
                                       b.y * (v[u].y / (1.f + __expf(-v[u].y))),
                                       b.z * (v[u].z / (1.f + __expf(-v[u].z))),
                                       b.w * (v[u].w / (1.f + __expf(-v[u].w))));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if ((it0 + u) * NT >= total) break;  // uniform across the CTA
            const int g = (it0 + u) * NT + threadIdx.x;
            const int pos = (np == 1 || g >= total) ? 0 : g / n4;
            const int f = g - pos * n4;
            uint8_t *hi = base + pos * pos_bytes;
            uint8_t *lo = hi + cols;
            float2 *rec = reinterpret_cast<float2 *>(hi + 2 * cols);
            uint32_t a = max(max(__float_as_uint(fabsf(v[u].x)), __float_as_uint(fabsf(v[u].y))),
                             max(__float_as_uint(fabsf(v[u].z)), __float_as_uint(fabsf(v[u].w))));
            a = max(a, __shfl_xor_sync(kFull, a, 1));
            a = max(a, __shfl_xor_sync(kFull, a, 2));
            a = max(a, __shfl_xor_sync(kFull, a, 4));
            // Power-of-two scale s = 2^e with |x| / s <= 32639: x * 2^-e is
            // exact, so dyadic inputs (small integers, k/2^n) stay exact.
            const bool bad = a >= 0x7f800000u;
            if (special != nullptr && g < total && (bad || (a != 0u && (a >> 23) < 27u))) *special = 1;
            const int ea = max((int)(a >> 23), 27);  // blocks below 2^-100 share 2^-114
            int e = ea - 127 - 14;
            float inv = __uint_as_float((uint32_t)(127 - e) << 23);
            if (__uint_as_float(a) * inv >= 32639.5f) {
                e += 1;
                inv *= 0.5f;
            }
            if (bad) inv = 0.f;
            const int q0 = __float2int_rn(v[u].x * inv), q1 = __float2int_rn(v[u].y * inv);
            const int q2 = __float2int_rn(v[u].z * inv), q3 = __float2int_rn(v[u].w * inv);
            const int h0 = (q0 + 128) >> 8, h1 = (q1 + 128) >> 8, h2 = (q2 + 128) >> 8, h3 = (q3 + 128) >> 8;
            const int l0 = q0 - (h0 << 8), l1 = q1 - (h1 << 8), l2 = q2 - (h2 << 8), l3 = q3 - (h3 << 8);
            const uint32_t hh = (uint32_t)(h0 & 0xff) | ((uint32_t)(h1 & 0xff) << 8) |
                                ((uint32_t)(h2 & 0xff) << 16) | ((uint32_t)(h3 & 0xff) << 24);
            const uint32_t ll = (uint32_t)(l0 & 0xff) | ((uint32_t)(l1 & 0xff) << 8) |
                                ((uint32_t)(l2 & 0xff) << 16) | ((uint32_t)(l3 & 0xff) << 24);
            int s4 = q0 + q1 + q2 + q3;
            s4 += __shfl_xor_sync(kFull, s4, 1);
            s4 += __shfl_xor_sync(kFull, s4, 2);
            if (g < total) {
                const int p = (4 * f) & ~15;
                const int si = Slices<FMT>::index(p, C);
                const int off = (si << 4) + ((4 * f) & 15);
                *reinterpret_cast<uint32_t *>(hi + off) = hh;
                *reinterpret_cast<uint32_t *>(lo + off) = ll;
                if ((f & 3) == 0) {
                    // s * sum is exact: s is a power of two, |sum| < 2^20
                    const float sc = bad ? __uint_as_float(0x7fc00000u) : __uint_as_float((uint32_t)(127 + e) << 23);
                    rec[si] = make_float2(sc, sc * (float)s4);
                }
            }
        }
    }
}

// ------------------------------------------------- per-format chunk code
//
// XR<N> holds the N x slices of one chunk in registers (loaded once, reused by
// every row the lane handles).  W<FMT> holds one row's chunk of weights:
// load() reads global memory (each piece a contiguous run across the warp),
// load_smem() reads a row staged in shared memory by the TMA pipeline, and
// dot() combines them.

template <int N> struct XR {
    uint4 h[N], l[N];
    float2 r[N];
};

template <int N>
__device__ __forceinline__ XR<N> load_xr(const XS &s, int C, int c)
{
    XR<N> x;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        x.h[j] = s.h(j, C, c);
        x.l[j] = s.l(j, C, c);
        x.r[j] = s.r(j, C, c);
    }
    return x;
}

__device__ __forceinline__ uint4 lds128(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}

__device__ __forceinline__ uint32_t lds16(uint32_t a)
{
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}

template <uint32_t FMT> struct W;

__device__ __forceinline__ int dot4(const uint4 &w, const uint4 &x, int acc)
{
    acc = dp4a(w.x, x.x, acc);
    acc = dp4a(w.y, x.y, acc);
    acc = dp4a(w.z, x.z, acc);
    return dp4a(w.w, x.w, acc);
}

template <> struct W<kQ8_0> {
    static constexpr int kSlices = 2;
    uint4 a, b;
    uint32_t d;
    __device__ __forceinline__ void zero() { a = b = make_uint4(0, 0, 0, 0); d = 0; }
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int c)
    {
        a = ld_stream(row + (c << 4));
        b = ld_stream(row + ((L.C + c) << 4));
        d = ld_stream16(row + L.off_a + 2 * c);
    }
    __device__ __forceinline__ void load_smem(uint32_t row, const Layout &L, int c)
    {
        a = lds128(row + (c << 4));
        b = lds128(row + ((L.C + c) << 4));
        d = lds16(row + L.off_a + 2 * c);
    }
    // Unpacked chunk: what dot() needs, computed once per chunk and reused
    // by every position of a batch.
    struct U {
        uint4 a, b;
        float d;
    };
    __device__ __forceinline__ U unpack() const { return U{a, b, f16_fast(d)}; }
    static __device__ __forceinline__ float dot_u(const U &u, const XR<2> &x)
    {
        const int ah = dot4(u.b, x.h[1], dot4(u.a, x.h[0], 0));
        const int al = dot4(u.b, x.l[1], dot4(u.a, x.l[0], 0));
        return (u.d * x.r[0].x) * (float)(ah * 256 + al);
    }
    // weights 32c.. of chunk (block) c: d * q
    template <typename XF>
    static __device__ __forceinline__ float dot_f32(const U &u, int c, const XF &xv)
    {
        const auto f = [&](uint32_t q) { return u.d * (float)(int8_t)q; };
        return dot16_f32(u.b, 32 * c + 16, f, xv, dot16_f32(u.a, 32 * c, f, xv, 0.f));
    }
    __device__ __forceinline__ float dot(const XR<2> &x) const { return dot_u(unpack(), x); }
};

// Spread bits 0..3 of v to bit 4 of bytes 0..3.
__device__ __forceinline__ uint32_t spread4(uint32_t v)
{
    return ((v & 0xfu) * 0x02040810u) & 0x10101010u;
}

template <> struct W<kQ5_0> {
    static constexpr int kSlices = 2;
    uint4 q;
    uint32_t qh, d;
    __device__ __forceinline__ void zero() { q = make_uint4(0, 0, 0, 0); qh = d = 0; }
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int c)
    {
        q = ld_stream(row + (c << 4));
        qh = ld_stream32(row + L.off_a + 4 * c);
        d = ld_stream16(row + L.off_b + 2 * c);
    }
    __device__ __forceinline__ void load_smem(uint32_t row, const Layout &L, int c)
    {
        q = lds128(row + (c << 4));
        qh = lds32(row + L.off_a + 4 * c);
        d = lds16(row + L.off_b + 2 * c);
    }
    struct U {
        uint4 lw, hw;
        float d;
    };
    __device__ __forceinline__ U unpack() const
    {
        // weights 4k..4k+3 from low nibbles, 16+4k.. from high nibbles; the
        // fifth bit of weight i is bit i of qh
        U u;
        u.lw = make_uint4((q.x & 0x0f0f0f0fu) | spread4(qh), (q.y & 0x0f0f0f0fu) | spread4(qh >> 4),
                          (q.z & 0x0f0f0f0fu) | spread4(qh >> 8), (q.w & 0x0f0f0f0fu) | spread4(qh >> 12));
        u.hw = make_uint4(((q.x >> 4) & 0x0f0f0f0fu) | spread4(qh >> 16), ((q.y >> 4) & 0x0f0f0f0fu) | spread4(qh >> 20),
                          ((q.z >> 4) & 0x0f0f0f0fu) | spread4(qh >> 24), ((q.w >> 4) & 0x0f0f0f0fu) | spread4(qh >> 28));
        u.d = f16_fast(d);
        return u;
    }
    static __device__ __forceinline__ float dot_u(const U &u, const XR<2> &x)
    {
        const int ah = dot4(u.hw, x.h[1], dot4(u.lw, x.h[0], 0));
        const int al = dot4(u.hw, x.l[1], dot4(u.lw, x.l[0], 0));
        return u.d * (x.r[0].x * (float)(ah * 256 + al) - 16.f * (x.r[0].y + x.r[1].y));
    }
    // weights 32c.. of block c: d * (v - 16)
    template <typename XF>
    static __device__ __forceinline__ float dot_f32(const U &u, int c, const XF &xv)
    {
        const auto f = [&](uint32_t v) { return u.d * (float)((int)v - 16); };
        return dot16_f32(u.hw, 32 * c + 16, f, xv, dot16_f32(u.lw, 32 * c, f, xv, 0.f));
    }
    __device__ __forceinline__ float dot(const XR<2> &x) const { return dot_u(unpack(), x); }
};

// Unsigned bytes of a times signed bytes of b, summed into c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ int dot4_us(const uint4 &w, const uint4 &x, int acc)
{
    acc = dp4a_us(w.x, x.x, acc);
    acc = dp4a_us(w.y, x.y, acc);
    acc = dp4a_us(w.z, x.z, acc);
    return dp4a_us(w.w, x.w, acc);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

template <> struct W<kQ4_K> {
    static constexpr int kSlices = 4;
    uint4 a, b, hdr;
    int g;
    __device__ __forceinline__ void zero() { a = b = hdr = make_uint4(0, 0, 0, 0); g = 0; }
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int c)
    {
        a = ld_stream(row + (c << 4));
        b = ld_stream(row + ((L.C + c) << 4));
        hdr = ld_stream(row + L.off_a + ((c >> 2) << 4));
        g = c & 3;
    }
    __device__ __forceinline__ void load_smem(uint32_t row, const Layout &L, int c)
    {
        a = lds128(row + (c << 4));
        b = lds128(row + ((L.C + c) << 4));
        hdr = lds128(row + L.off_a + ((c >> 2) << 4));
        g = c & 3;
    }
    // Weights of sub-block 2g (low nibbles, la/lb) and of sub-block 2g+1
    // (high nibbles left in place, ua/ub: 16 times the value, which the
    // unsigned-by-signed dp4a sums exactly; s1 carries the 1/16).
    struct U {
        uint4 la, lb, ua, ub;
        float s0, m0, s1, m1;  // d * sc and dmin * m of sub-blocks 2g and 2g+1 (s1 over 16)
    };
    __device__ __forceinline__ U unpack() const
    {
        U u;
        u.la = make_uint4(a.x & 0x0f0f0f0fu, a.y & 0x0f0f0f0fu, a.z & 0x0f0f0f0fu, a.w & 0x0f0f0f0fu);
        u.lb = make_uint4(b.x & 0x0f0f0f0fu, b.y & 0x0f0f0f0fu, b.z & 0x0f0f0f0fu, b.w & 0x0f0f0f0fu);
        u.ua = make_uint4(a.x & 0xf0f0f0f0u, a.y & 0xf0f0f0f0u, a.z & 0xf0f0f0f0u, a.w & 0xf0f0f0f0u);
        u.ub = make_uint4(b.x & 0xf0f0f0f0u, b.y & 0xf0f0f0f0u, b.z & 0xf0f0f0f0u, b.w & 0xf0f0f0f0u);
        // 6-bit scale / min of sub-blocks j = 2g, 2g+1 from the 12 bytes
        // b[0..11] = hdr.y, hdr.z, hdr.w (src/quantization.cpp:351-378).
        // j < 4: sc = b[j] & 63, m = b[j+4] & 63.  j >= 4: sc = (b[j+4] & 15) |
        // (b[j-4] >> 6) << 4, m = (b[j+4] >> 4) | (b[j] >> 6) << 4.  With
        // h = g & 1, P gathers bytes (y[2h], y[2h+1], z[2h], z[2h+1]) and Q
        // (w[2h], w[2h+1], w[2h], w[2h+1]); the result's bytes are
        // (sc_2g, sc_2g+1, m_2g, m_2g+1).  The selectors and masks depend only
        // on the lane's g.
        const bool lo = g < 2;
        const uint32_t P = prmt(hdr.y, hdr.z, (g & 1) ? 0x7632u : 0x5410u);
        const uint32_t Q = prmt(hdr.w, hdr.w, (g & 1) ? 0x3232u : 0x1010u);
        const uint32_t v = (P & (lo ? 0x3f3f3f3fu : 0u)) | ((P >> 2) & (lo ? 0u : 0x30303030u)) |
                           (Q & (lo ? 0u : 0x00000f0fu)) | ((Q >> 4) & (lo ? 0u : 0x0f0f0000u));
        const float d = f16_fast(hdr.x), dmin = f16_fast(hdr.x >> 16);
        u.s0 = d * (float)(v & 0xffu);
        u.s1 = (d * (float)((v >> 8) & 0xffu)) * 0.0625f;
        u.m0 = dmin * (float)((v >> 16) & 0xffu);
        u.m1 = dmin * (float)(v >> 24);
        return u;
    }
    static __device__ __forceinline__ float dot_u(const U &u, const XR<4> &x)
    {
        const int ah0 = dot4_us(u.lb, x.h[1], dot4_us(u.la, x.h[0], 0));
        const int al0 = dot4_us(u.lb, x.l[1], dot4_us(u.la, x.l[0], 0));
        const int ah1 = dot4_us(u.ub, x.h[3], dot4_us(u.ua, x.h[2], 0));
        const int al1 = dot4_us(u.ub, x.l[3], dot4_us(u.ua, x.l[2], 0));
        const float v0 = u.s0 * (x.r[0].x * (float)(ah0 * 256 + al0)) - u.m0 * (x.r[0].y + x.r[1].y);
        const float v1 = u.s1 * (x.r[2].x * (float)(ah1 * 256 + al1)) - u.m1 * (x.r[2].y + x.r[3].y);
        return v0 + v1;
    }
    __device__ __forceinline__ float dot(const XR<4> &x) const { return dot_u(unpack(), x); }
    // weights 64c.. of chunk c (sub-blocks 2g, 2g+1): d sc q - dmin m
    template <typename XF>
    static __device__ __forceinline__ float dot_f32(const U &u, int c, const XF &xv)
    {
        const float s1 = u.s1 * 16.f;  // the high-nibble bytes hold 16 q
        const auto f0 = [&](uint32_t q) { return u.s0 * (float)q - u.m0; };
        const auto f1 = [&](uint32_t q) { return s1 * (float)(q >> 4) - u.m1; };
        float acc = dot16_f32(u.la, 64 * c, f0, xv, 0.f);
        acc = dot16_f32(u.lb, 64 * c + 16, f0, xv, acc);
        acc = dot16_f32(u.ua, 64 * c + 32, f1, xv, acc);
        return dot16_f32(u.ub, 64 * c + 48, f1, xv, acc);
    }
};

// Signed byte B of v as an int, in one byte-permute (sign-replicating
// selector nibbles).
template <int B>
__device__ __forceinline__ int sbyte(uint32_t v)
{
    int r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(v), "n"(((8 | B) << 12) | ((8 | B) << 8) | ((8 | B) << 4) | B));
    return r;
}

template <> struct W<kQ6_K> {
    static constexpr int kSlices = 4;
    uint4 a, b, u;
    uint32_t sc, d;
    __device__ __forceinline__ void zero() { a = b = u = make_uint4(0, 0, 0, 0); sc = d = 0; }
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int c)
    {
        a = ld_stream(row + (c << 4));
        b = ld_stream(row + ((L.C + c) << 4));
        u = ld_stream(row + ((2 * L.C + c) << 4));
        sc = ld_stream32(row + L.off_a + 4 * c);
        d = ld_stream16(row + L.off_b + 2 * (c >> 2));
    }
    __device__ __forceinline__ void load_smem(uint32_t row, const Layout &L, int c)
    {
        a = lds128(row + (c << 4));
        b = lds128(row + ((L.C + c) << 4));
        u = lds128(row + ((2 * L.C + c) << 4));
        sc = lds32(row + L.off_a + 4 * c);
        d = lds16(row + L.off_b + 2 * (c >> 2));
    }
    struct U {
        uint4 w0, w1, w2, w3;
        float s0, s1, s2, s3, d;
    };
    __device__ __forceinline__ U unpack() const
    {
        // 6-bit values 0..63 per region (src/quantization.cpp:559-586)
        U r;
        r.w0 = make_uint4((a.x & 0x0f0f0f0fu) | ((u.x << 4) & 0x30303030u), (a.y & 0x0f0f0f0fu) | ((u.y << 4) & 0x30303030u),
                          (a.z & 0x0f0f0f0fu) | ((u.z << 4) & 0x30303030u), (a.w & 0x0f0f0f0fu) | ((u.w << 4) & 0x30303030u));
        r.w1 = make_uint4((b.x & 0x0f0f0f0fu) | ((u.x << 2) & 0x30303030u), (b.y & 0x0f0f0f0fu) | ((u.y << 2) & 0x30303030u),
                          (b.z & 0x0f0f0f0fu) | ((u.z << 2) & 0x30303030u), (b.w & 0x0f0f0f0fu) | ((u.w << 2) & 0x30303030u));
        r.w2 = make_uint4(((a.x >> 4) & 0x0f0f0f0fu) | (u.x & 0x30303030u), ((a.y >> 4) & 0x0f0f0f0fu) | (u.y & 0x30303030u),
                          ((a.z >> 4) & 0x0f0f0f0fu) | (u.z & 0x30303030u), ((a.w >> 4) & 0x0f0f0f0fu) | (u.w & 0x30303030u));
        r.w3 = make_uint4(((b.x >> 4) & 0x0f0f0f0fu) | ((u.x >> 2) & 0x30303030u),
                          ((b.y >> 4) & 0x0f0f0f0fu) | ((u.y >> 2) & 0x30303030u),
                          ((b.z >> 4) & 0x0f0f0f0fu) | ((u.z >> 2) & 0x30303030u),
                          ((b.w >> 4) & 0x0f0f0f0fu) | ((u.w >> 2) & 0x30303030u));
        r.s0 = (float)sbyte<0>(sc);
        r.s1 = (float)sbyte<1>(sc);
        r.s2 = (float)sbyte<2>(sc);
        r.s3 = (float)sbyte<3>(sc);
        r.d = f16_fast(d);
        return r;
    }
    static __device__ __forceinline__ float dot_u(const U &r, const XR<4> &x)
    {
        const int A0 = dot4(r.w0, x.h[0], 0) * 256 + dot4(r.w0, x.l[0], 0);
        const int A1 = dot4(r.w1, x.h[1], 0) * 256 + dot4(r.w1, x.l[1], 0);
        const int A2 = dot4(r.w2, x.h[2], 0) * 256 + dot4(r.w2, x.l[2], 0);
        const int A3 = dot4(r.w3, x.h[3], 0) * 256 + dot4(r.w3, x.l[3], 0);
        float acc = r.s0 * (x.r[0].x * (float)A0 - 32.f * x.r[0].y);
        acc += r.s1 * (x.r[1].x * (float)A1 - 32.f * x.r[1].y);
        acc += r.s2 * (x.r[2].x * (float)A2 - 32.f * x.r[2].y);
        acc += r.s3 * (x.r[3].x * (float)A3 - 32.f * x.r[3].y);
        return r.d * acc;
    }
    // chunk c = 4 sb + 2 g + h holds weights 256 sb + 128 g + 32 r + 16 h + o:
    // d * sc_r * (q - 32)
    template <typename XF>
    static __device__ __forceinline__ float dot_f32(const U &r, int c, const XF &xv)
    {
        const int base = 256 * (c >> 2) + 128 * ((c >> 1) & 1) + 16 * (c & 1);
        const auto f0 = [&](uint32_t q) { return r.d * r.s0 * (float)((int)q - 32); };
        const auto f1 = [&](uint32_t q) { return r.d * r.s1 * (float)((int)q - 32); };
        const auto f2 = [&](uint32_t q) { return r.d * r.s2 * (float)((int)q - 32); };
        const auto f3 = [&](uint32_t q) { return r.d * r.s3 * (float)((int)q - 32); };
        float acc = dot16_f32(r.w0, base, f0, xv, 0.f);
        acc = dot16_f32(r.w1, base + 32, f1, xv, acc);
        acc = dot16_f32(r.w2, base + 64, f2, xv, acc);
        return dot16_f32(r.w3, base + 96, f3, xv, acc);
    }
    __device__ __forceinline__ float dot(const XR<4> &x) const { return dot_u(unpack(), x); }
};

// ------------------------------------------------ fp32 rows (rare path)
//
// When x holds a NaN/Inf or a tiny block, a CTA computes its rows in fp32:
// each weight dequantized as the reference does (src/quantization.cpp:54-67,
// 161-184, 380-409, 588-615) times the float x, so Inf and NaN propagate as in
// the reference's loops and tiny magnitudes keep their bits.  xv(k) returns
// element k of the (prologue-transformed) x.

template <int K>
__device__ __forceinline__ uint32_t byte_at(const uint4 &v)
{
    const uint32_t w = K < 4 ? v.x : K < 8 ? v.y : K < 12 ? v.z : v.w;
    return (w >> (8 * (K & 3))) & 0xffu;
}

// Element k of position p's x as the fused prologue forms it (the fp32 rows).
struct XVal {
    const float *x;
    int pre;
    float denom;
    const float *aux;
    __device__ __forceinline__ float operator()(int k) const
    {
        const float v = __ldg(x + k);
        if (pre == kPreRmsNorm) return (v / denom) * __ldg(aux + k);
        if (pre == kPreSwiGlu) return __ldg(aux + k) * (v / (1.f + expf(-v)));
        return v;
    }
};

// sum over the 16 bytes of v of f(byte, k) * x[base + k]
template <typename F, typename XF>
__device__ __forceinline__ float dot16_f32(const uint4 &v, int base, const F &f, const XF &xv, float acc)
{
#define QMV_DOT16_STEP(K) acc = fmaf(f(byte_at<K>(v)), xv(base + (K)), acc);
    QMV_DOT16_STEP(0) QMV_DOT16_STEP(1) QMV_DOT16_STEP(2) QMV_DOT16_STEP(3)
    QMV_DOT16_STEP(4) QMV_DOT16_STEP(5) QMV_DOT16_STEP(6) QMV_DOT16_STEP(7)
    QMV_DOT16_STEP(8) QMV_DOT16_STEP(9) QMV_DOT16_STEP(10) QMV_DOT16_STEP(11)
    QMV_DOT16_STEP(12) QMV_DOT16_STEP(13) QMV_DOT16_STEP(14) QMV_DOT16_STEP(15)
#undef QMV_DOT16_STEP
    return acc;
}

// fp32 rows [r0, r1) of y (the rare path): a warp per row, lanes over its
// chunks read from global memory; y[row] = dot (+ add[row]).  Returns the
// calling thread's best argmax key of the rows it wrote.  Not inlined: kept
// out of the GEMV kernels' code it would otherwise slow down (measured).
template <uint32_t FMT>
__device__ __noinline__ unsigned long long fp32_rows(const Layout &L, const uint8_t *__restrict__ w, int r0, int r1, int warp,
                                        int nwarps, const XVal &xv, float *y, const float *add, bool want_key,
                                        int index_base)
{
    const int lane = threadIdx.x & 31;
    unsigned long long best = 0ull;
    for (int row = r0 + warp; row < r1; row += nwarps) {
        float acc = 0.f;
        for (int c = lane; c < L.C; c += 32) {
            W<FMT> wv;
            wv.load(w + (uint64_t)row * L.row_stride, L, c);
            acc += W<FMT>::dot_f32(wv.unpack(), c, xv);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
        if (lane == 0) {
            const float out = add != nullptr ? acc + add[row] : acc;
            y[row] = out;
            if (want_key) best = max_ull(best, make_key(out, index_base + row));
        }
    }
    return best;
}

// ------------------------------------------------------- GEMV (loads)
//
// Direct-load form (used when the TMA stages below do not fit, e.g. very
// long rows).  Persistent grid.  A warp owns whole row tiles: TPT lanes (16
// or 32) per group, 32/TPT groups per warp, R rows per group, so a warp tile
// is (32/TPT)*R consecutive rows.  Warp tiles are dealt round-robin over every
// warp of the grid.  Within a tile the group's lanes stride over the chunks
// of its rows; one x slice set serves R rows.  The next item's weights are
// loaded before the current item is computed (one-deep register prefetch),
// and the only synchronisation is a shuffle reduction in a fixed order, so
// results are deterministic.

template <uint32_t FMT, int TPT, int R>
__global__ void __launch_bounds__(kThreads)
gemv_kernel(Layout L, const uint8_t *__restrict__ w, const float *__restrict__ x,
            float *__restrict__ y, ArgmaxOut am, int want_argmax)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long kscratch[kThreads / 32];
    __shared__ int special;
    constexpr int NSL = W<FMT>::kSlices;

    const int C = L.C;
    if (threadIdx.x == 0) special = 0;
    __syncthreads();
    quantize_x<FMT>(x, L.cols, C, smem, 1, 0, kPreNone, 1.f, nullptr, &special);
    __syncthreads();
    const bool f32 = *(volatile int *)&special != 0;
    const XS s = xs_view(smem, L.cols);

    constexpr int GPW = 32 / TPT;
    constexpr int WR = GPW * R;
    const int lane = threadIdx.x & 31;
    const int grp = lane / TPT, gl = lane % TPT;
    const int wg = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    const int wtot = gridDim.x * (kThreads / 32);
    const int NI = (C + TPT - 1) / TPT;
    const int tiles = (L.rows + WR - 1) / WR;
    const int my_tiles = wg < tiles ? (tiles - 1 - wg) / wtot + 1 : 0;
    const int n_items = my_tiles * NI;

    unsigned long long best = 0ull;
    W<FMT> bufa[R], bufb[R];
    float acc[R];
#pragma unroll
    for (int i = 0; i < R; ++i) acc[i] = 0.f;

    // Item k = (tile t, chunk iteration it); both advance incrementally.
    auto load_item = [&](int t, int it, W<FMT> (&dst)[R]) {
        const int c = it * TPT + gl;
        const int row0 = t * WR + grp * R;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            if (c < C && row0 + i < L.rows)
                dst[i].load(w + (uint64_t)(row0 + i) * L.row_stride, L, c);
            else
                dst[i].zero();
        }
    };
    // Compute item (t, it) from `use` while `pre` receives item k+1.
    auto step = [&](int k, int &t, int &it, W<FMT> (&use)[R], W<FMT> (&pre)[R]) {
        int nt = t, nit = it + 1;
        if (nit == NI) {
            nit = 0;
            nt += wtot;
        }
        if (k + 1 < n_items) load_item(nt, nit, pre);
        const int c = it * TPT + gl;
        const int row0 = t * WR + grp * R;
        if (c < C) {
            const XR<NSL> xr = load_xr<NSL>(s, C, c);
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] += use[i].dot(xr);
        }
        if (it == NI - 1) {
#pragma unroll
            for (int i = 0; i < R; ++i) {
#pragma unroll
                for (int o = TPT / 2; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
            }
            float out = 0.f;
#pragma unroll
            for (int i = 0; i < R; ++i)
                if (gl == i) out = acc[i];
            if (gl < R && row0 + gl < L.rows) {
                y[row0 + gl] = out;
                if (want_argmax) best = max_ull(best, make_key(out, am.index_base + row0 + gl));
            }
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] = 0.f;
        }
        t = nt;
        it = nit;
    };

    if (f32) {
        // special x: every row of the grid in fp32, a warp per row
        best = fp32_rows<FMT>(L, w, 0, L.rows, wg, wtot, XVal{x, kPreNone, 1.f, nullptr}, y, nullptr,
                              want_argmax != 0, am.index_base);
    } else {
        int t = wg, it = 0;
        if (n_items > 0) load_item(t, it, bufa);
        for (int k = 0; k < n_items; k += 2) {
            step(k, t, it, bufa, bufb);
            if (k + 1 < n_items) step(k + 1, t, it, bufb, bufa);
        }
    }
    if (want_argmax) {
        best = block_max_key(best, kscratch);
        finish_argmax(best, am, kscratch);
    }
}

// --------------------------------------------------- GEMV (TMA pipeline)
//
// One CTA per SM owns a contiguous range of rows, which is one contiguous
// byte range of the resident tensor.  A producer warp streams it into a ring
// of NS shared-memory stages with cp.async.bulk (1-D TMA, no multicast),
// each stage holding kConsumerWarps * R rows and completing on an mbarrier
// with its byte count.  Consumer warps each take R rows of a stage; their
// lanes stride over the chunks, loading the x slices of a chunk once for the
// R rows, then release the stage through an "empty" mbarrier.  Weights are
// read from shared memory with conflict-free 128-bit loads (chunk-major rows).
//
// Every mbarrier wait is bounded by a globaltimer deadline: on expiry the
// waiting thread sets a bit in g_status, stops issuing work, and the producer
// still waits (again bounded) for the copies it has in flight before the CTA
// exits.

constexpr int kMaxConsumerWarps = 16;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ unsigned int g_status;
enum : unsigned int { kStatusConsumerTimeout = 1u, kStatusProducerTimeout = 2u, kStatusDrainTimeout = 4u };

// An expired wait sets its bit in the device-wide word and, when the launch
// carries one, in the calling thread's own word (a mapped host word of the
// drop-in calls, written with a plain store: host memory need not support
// device atomics), so a concurrent caller's clean call is not failed by
// another's timeout.
__device__ __forceinline__ void report_status(unsigned int *call_status, unsigned int bit)
{
    atomicOr(&g_status, bit);
    if (call_status != nullptr) *(volatile unsigned int *)call_status = *(volatile unsigned int *)call_status | bit;
}

__device__ __forceinline__ unsigned long long globaltimer()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try(bar, parity)) return true;
        if ((n & 63u) == 0u && globaltimer() - t0 > kWaitLimitNs) return false;
    }
}

// The same wait for threads that have nothing else to do: each try suspends
// the thread (up to 0.5 us, or until the phase completes) instead of
// re-issuing, so a waiting producer or MMA thread does not take issue slots
// from the warps sharing its scheduler.
__device__ __forceinline__ bool mbar_try_idle(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(500u)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_idle(uint32_t bar, uint32_t parity)
{
    if (mbar_try_idle(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (mbar_try_idle(bar, parity)) return true;
        if (globaltimer() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Prefetch of the L2 line holding p (a valid address).
__device__ __forceinline__ void prefetch_line_l2(const void *p)
{
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share (of ncta) of the fused prefetch ranges.
__device__ __forceinline__ void prefetch_share(const Fuse &fu, int cta, int ncta)
{
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        if (fu.pf[i] == nullptr || fu.pf_bytes[i] == 0) continue;
        const uint64_t B = fu.pf_bytes[i];
        const uint64_t b0 = (B * (uint64_t)cta / (uint64_t)ncta) & ~15ull;
        const uint64_t b1 = cta + 1 == ncta ? (B & ~15ull) : ((B * (uint64_t)(cta + 1) / (uint64_t)ncta) & ~15ull);
        for (uint64_t off = b0; off < b1; off += 65536u)
            prefetch_l2(fu.pf[i] + off, (uint32_t)(b1 - off < 65536u ? b1 - off : 65536u));
    }
}

struct TmaPlan {
    uint32_t x_bytes;      // quantized x, rounded to 128
    uint32_t stage_bytes;  // rows_per_stage * row_stride, rounded to 128
    int rows_per_stage;    // CW * R
    int stages;            // NS
    int consumer_warps;    // CW
    int rows_per_warp;     // R
    int np;                // positions (1: GEMV; up to the kernel's NP: batched)
    int split;             // warps per row (2: long rows, see gemv_tma_kernel)
    unsigned int *status;  // the calling thread's status word, or null
};

// NP > 1: the batched form for up to NP positions (x holds P.np rows of
// cols floats, y P.np rows of L.rows); each staged weight chunk is unpacked
// once per row and applied to every position.  No argmax or exchange there.
// SPLIT = 2 (long rows, where only a few rows fit a stage): two warps share
// each row, taking alternate 32-chunk blocks; the second warp's sum reaches
// the first through shared memory, handed over with a pair of mbarriers per
// stage parity (bounded waits, like every other wait here).
// The statically sized shared state of one GEMV CTA.
struct TmaShared {
    // full: per stage and row slot (the R rows of one consumer warp, or of a
    // warp pair in the split-row plan), so a warp starts as soon as its own
    // rows have landed; empty: per stage; pbar: pfull[2] | pfree[2]
    unsigned long long full[8][kMaxConsumerWarps];
    unsigned long long empty[8];
    unsigned long long pbar[4];
    unsigned long long kscratch[kMaxConsumerWarps + 1];
    float partial[2][kMaxConsumerWarps];
    float sumsq[kMaxConsumerWarps];
    int special;  // x holds a NaN/Inf or tiny block: rows in fp32
};


// One CTA (number cta of ncta sharing the matrix) of the TMA GEMV; smem is
// the dynamic shared memory (quantized x, then the stage ring).
// RARE: compile the fp32 rows of a special x (the paired gate/up launch of
// the decode step leaves them out: there any non-finite value fails the step).
template <uint32_t FMT, int CW, int R, int NP = 1, int SPLIT = 1, bool RARE = true>
__device__ __forceinline__ void gemv_tma_body(uint8_t *smem, TmaShared &sh, int cta, int ncta, const Layout &L,
                                              const uint8_t *__restrict__ w, const float *__restrict__ x,
                                              float *__restrict__ y_, const ArgmaxOut &am, int want_argmax,
                                              const TmaPlan &P, const Exchange &ex, const Fuse &fu)
{
    static_assert(R * NP <= 32, "one lane per (row, position) output");
    static_assert(SPLIT == 1 || (SPLIT == 2 && R == 1 && NP == 1 && CW % 2 == 0), "split rows: one row per warp pair");
    float *y = y_;
    constexpr int kConsumerWarps = CW;
    constexpr int NSL = W<FMT>::kSlices;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = L.C;
    const int NS = P.stages;
    const uint32_t stage0 = (uint32_t)__cvta_generic_to_shared(smem + P.x_bytes);
    const uint32_t full0 = (uint32_t)__cvta_generic_to_shared(&sh.full[0][0]);
    const uint32_t empty0 = (uint32_t)__cvta_generic_to_shared(&sh.empty[0]);
    const uint32_t pbar0 = (uint32_t)__cvta_generic_to_shared(&sh.pbar[0]);
    constexpr int NSLOT = CW / SPLIT;  // row slots per stage, R rows each
    // the full barrier of stage sidx, row slot j
    auto full = [&](int sidx, int j) { return full0 + 8u * (uint32_t)(sidx * kMaxConsumerWarps + j); };

    const int r0 = (int)((long long)L.rows * cta / ncta);
    const int r1 = (int)((long long)L.rows * (cta + 1) / ncta);
    const int SR = P.rows_per_stage;
    const int n_stages = (r1 - r0 + SR - 1) / SR;
    // Programmatic dependent launch: the next launch in the stream may start
    // now; it only streams weights until its griddepcontrol.wait, and this
    // grid touches x, y, the workspace and the exchange buffers only after its
    // own wait (i.e. after the previous grid has completed).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) {
            for (int j = 0; j < NSLOT; ++j) mbar_init(full(i, j), 1u);
            mbar_init(empty0 + 8u * i, (uint32_t)kConsumerWarps);
        }
        for (int i = 0; i < 4; ++i) mbar_init(pbar0 + 8u * i, (uint32_t)(kConsumerWarps / 2));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.special = 0;
    }
    __syncthreads();

    unsigned long long best = 0ull;
    if (warp == kConsumerWarps) {
        // ---------------- producer: lane j copies row slot j of each stage
        int issued = 0;
        bool ok = true;
        for (int k = 0; k < n_stages; ++k) {
            const int sidx = k % NS;
            if (k >= NS) {
                const bool freed = mbar_wait(empty0 + 8u * sidx, (uint32_t)((k / NS - 1) & 1));
                if (!__all_sync(kFull, freed)) {
                    if (lane == 0) report_status(P.status, kStatusProducerTimeout);
                    ok = false;
                    break;
                }
            }
            if (lane < NSLOT) {
                const int rows_k = min(SR, r1 - (r0 + k * SR));
                const int lr = lane * R, nr = min(R, rows_k - lr);
                const uint32_t bar = full(sidx, lane);
                if (nr > 0) {
                    const uint32_t bytes = (uint32_t)nr * (uint32_t)L.row_stride;
                    mbar_expect_tx(bar, bytes);
                    const uint8_t *src = w + (uint64_t)(r0 + k * SR + lr) * L.row_stride;
                    const uint32_t dst = stage0 + (uint32_t)sidx * P.stage_bytes + (uint32_t)lr * (uint32_t)L.row_stride;
                    for (uint32_t off = 0; off < bytes; off += 32768u)
                        bulk_g2s(dst + off, src + off, min(32768u, bytes - off), bar);
                } else {
                    mbar_arrive(bar);  // a slot past the last row: its phase completes at once
                }
            }
            ++issued;
        }
        if (!ok && lane < NSLOT) {
            // drain: every issued copy must land before the CTA exits
            for (int k = max(0, issued - NS); k < issued; ++k) {
                if (!mbar_wait(full(k % NS, lane), (uint32_t)((k / NS) & 1))) {
                    report_status(P.status, kStatusDrainTimeout);
                    break;
                }
            }
        }
        if (ok && lane == 0) prefetch_share(fu, (int)blockIdx.x, (int)gridDim.x);
        __syncwarp();
        asm volatile("griddepcontrol.wait;" ::: "memory");
    } else {
        // ---------------- consumers
        // The RMSNorm weights and the epilogue's addend rows of this CTA do
        // not depend on the previous launch (the addend is a bias, or the
        // residual stream, whose lines are then simply in L2 already): bring
        // their lines into L2 while the previous launch finishes.
        if (NP == 1) {
            if (fu.pre == kPreRmsNorm)
                for (int i = threadIdx.x * 32; i < L.cols; i += CW * 32 * 32) prefetch_line_l2(fu.norm + i);
            if (fu.add != nullptr)
                for (int i = r0 + threadIdx.x * 32; i < r1; i += CW * 32 * 32) prefetch_line_l2(fu.add + i);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (ex.world > 1)  // this rank's slot in this epoch's parity region
            y = ex.logits[exchange_epoch(ex) & 1u][ex.rank] + (size_t)ex.rank * ex.slot_rows;
        const size_t xb = xs_bytes(L.cols);
        // One pass over x: the RMSNorm prologue quantizes x * norm and scales
        // the row sums by 1 / sqrt(mean(x^2) + eps), whose sum of squares is
        // gathered in the same pass.
        const bool rms = NP == 1 && fu.pre == kPreRmsNorm;
        const int pre = NP == 1 ? (rms ? kPreScale : fu.pre) : kPreNone;
        const float *aux = fu.pre == kPreRmsNorm ? fu.norm : fu.up;
        float ss = 0.f;
        quantize_x<FMT, CW * 32>(x, L.cols, C, smem, NP == 1 ? 1 : P.np, xb, pre, 1.f, aux,
                                 RARE ? &sh.special : nullptr, &ss);
        if (rms) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
            if (lane == 0) sh.sumsq[warp] = ss;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
        float denom = 1.f, rscale = 1.f;
        if (rms) {
            ss = 0.f;
            for (int i = 0; i < CW; ++i) ss += sh.sumsq[i];
            denom = sqrtf(ss / (float)L.cols + fu.eps);
            rscale = 1.f / denom;
        }
        const bool f32 = *(volatile int *)&sh.special != 0;  // uniform over the CTA
        const XS s = xs_view(smem, L.cols);
        const int NI = (C + 32 * SPLIT - 1) / (32 * SPLIT);
        const int rw = warp % (CW / SPLIT), half = warp / (CW / SPLIT);  // row slot, chunk half
        if (RARE && f32) {
            // special x: consume the stages (the producer must finish), then
            // this CTA's rows in fp32 from global memory (every position of a
            // batch)
            for (int k = 0; k < n_stages; ++k) {
                if (!mbar_wait(full(k % NS, rw), (uint32_t)((k / NS) & 1))) {
                    report_status(P.status, kStatusConsumerTimeout);
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8u * (k % NS));
            }
            if constexpr (NP == 1) {
                best = fp32_rows<FMT>(L, w, r0, r1, warp, CW, XVal{x, fu.pre, denom, aux}, y, fu.add,
                                      want_argmax != 0, am.index_base);
            } else {
                for (int p = 0; p < P.np; ++p)
                    fp32_rows<FMT>(L, w, r0, r1, warp, CW, XVal{x + (size_t)p * L.cols, kPreNone, 1.f, nullptr},
                                   y + (size_t)p * L.rows, nullptr, false, 0);
            }
        } else
        for (int k = 0; k < n_stages; ++k) {
            const int sidx = k % NS;
            if (!mbar_wait(full(sidx, rw), (uint32_t)((k / NS) & 1))) {
                report_status(P.status, kStatusConsumerTimeout);
                break;
            }
            const int base_row = r0 + k * SR;
            const int rows_k = min(SR, r1 - base_row);
            const uint32_t sbase = stage0 + (uint32_t)sidx * P.stage_bytes;
            float acc[R][NP];
#pragma unroll
            for (int i = 0; i < R; ++i) {
#pragma unroll
                for (int p = 0; p < NP; ++p) acc[i][p] = 0.f;
            }
            const int lr0 = rw * R;
            if (lr0 < rows_k) {
                for (int it = 0; it < NI; ++it) {
                    const int c = (it * SPLIT + half) * 32 + lane;
                    if (c < C) {
                        // All R rows are loaded without a row guard: the stage
                        // buffer holds CW * R rows, so rows past rows_k read
                        // in-bounds (stale) bytes whose sums are never written.
                        W<FMT> wv[R];
#pragma unroll
                        for (int i = 0; i < R; ++i)
                            wv[i].load_smem(sbase + (uint32_t)(lr0 + i) * (uint32_t)L.row_stride, L, c);
                        if constexpr (NP == 1) {
                            const XR<NSL> xr = load_xr<NSL>(s, C, c);
#pragma unroll
                            for (int i = 0; i < R; ++i) acc[i][0] += wv[i].dot(xr);
                        } else {
                            typename W<FMT>::U u[R];
#pragma unroll
                            for (int i = 0; i < R; ++i) u[i] = wv[i].unpack();
#pragma unroll
                            for (int p = 0; p < NP; ++p) {
                                if (p < P.np) {
                                    const XR<NSL> xr = load_xr<NSL>(xs_view(smem + p * xb, L.cols), C, c);
#pragma unroll
                                    for (int i = 0; i < R; ++i) acc[i][p] += W<FMT>::dot_u(u[i], xr);
                                }
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8u * sidx);
#pragma unroll
            for (int i = 0; i < R; ++i) {
#pragma unroll
                for (int p = 0; p < NP; ++p) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) acc[i][p] += __shfl_xor_sync(kFull, acc[i][p], o);
                }
            }
            if constexpr (SPLIT == 2) {
                // buffer pb of the partial sums carries stages k = pb (mod 2)
                const int pb = k & 1;
                const uint32_t pfull = pbar0 + 8u * pb, pfree = pbar0 + 8u * (2 + pb);
                bool okp = true;
                if (half == 1) {
                    // free once the partners have read stage k - 2
                    if (k >= 2) okp = mbar_wait(pfree, (uint32_t)(((k >> 1) - 1) & 1));
                    if (okp && lane == 0) sh.partial[pb][rw] = acc[0][0];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(pfull);
                } else {
                    okp = mbar_wait(pfull, (uint32_t)((k >> 1) & 1));
                    if (okp) acc[0][0] += sh.partial[pb][rw];
                    __syncwarp();
                    if (lane == 0) mbar_arrive(pfree);
                }
                if (!__all_sync(kFull, okp)) {
                    if (lane == 0) report_status(P.status, kStatusConsumerTimeout);
                    break;
                }
            }
            // lane j writes row lr0 + j / NP, position j % NP
            float out = 0.f;
#pragma unroll
            for (int i = 0; i < R; ++i) {
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    if (lane == i * NP + p) out = acc[i][p];
            }
            const int oi = lane / NP, op = lane % NP;
            if (half == 0 && lane < R * NP && lr0 + oi < rows_k && op < P.np) {
                const int row = base_row + lr0 + oi;
                out *= rscale;
                if (fu.add != nullptr) out += fu.add[(size_t)op * L.rows + row];
                y[(size_t)op * L.rows + row] = out;
                if (NP == 1 && want_argmax) best = max_ull(best, make_key(out, am.index_base + row));
            }
        }
    }
    if (ex.world > 1) {
        // this CTA's rows of y are written (block_max_key synchronizes first)
        best = block_max_key(best, sh.kscratch);
        const unsigned int epoch = exchange_epoch(ex);
        const int par = (int)(epoch & 1u);
        exchange_send(ex, par, epoch, ex.logits[par][ex.rank] + (size_t)ex.rank * ex.slot_rows, r0, r1, best);
        // the rank's last CTA collects
        __shared__ int is_last;
        unsigned int *counter = reinterpret_cast<unsigned int *>(am.workspace);
        if (threadIdx.x == 0) {
            __threadfence();
            is_last = atomicAdd(counter, 1u) == gridDim.x - 1u;
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        if (threadIdx.x == 0) *counter = 0u;
        exchange_collect(ex, par, epoch, am.key, sh.kscratch);
        return;
    }
    if (want_argmax) {
        best = block_max_key(best, sh.kscratch);
        finish_argmax(best, am, sh.kscratch);
    }
}

// MINB = 2: the register-capped instance of the shared plan, whose CTA
// leaves registers and shared memory for one CTA of the next launch on the
// same SM (programmatic dependent launch then streams that launch's first
// stages while this one finishes).
template <uint32_t FMT, int CW, int R, int NP = 1, int SPLIT = 1, int MINB = 1>
__global__ void __launch_bounds__((CW + 1) * 32, MINB)
gemv_tma_kernel(Layout L, const uint8_t *__restrict__ w, const float *__restrict__ x,
                float *__restrict__ y, ArgmaxOut am, int want_argmax, TmaPlan P, Exchange ex, Fuse fu)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TmaShared sh;
    gemv_tma_body<FMT, CW, R, NP, SPLIT>(smem, sh, (int)blockIdx.x, (int)gridDim.x, L, w, x, y, am, want_argmax, P,
                                         ex, fu);
}

// Two matrices with one input in one launch (the decode step's gate and up
// projections when their formats differ): CTAs [0, ctas0) take matrix 0, the
// rest matrix 1, each with its own plan; both read x through the same
// prologue (fu) and write their own output.
struct GemvPair {
    Layout L[2];
    const uint8_t *w[2];
    float *y[2];
    TmaPlan P[2];
    int ctas0;
};

template <uint32_t FA, uint32_t FB, int CW, int R>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
gemv_pair_kernel(GemvPair pr, const float *__restrict__ x, Fuse fu)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ TmaShared sh;
    const ArgmaxOut none{nullptr, nullptr, 0};
    const Exchange solo{};
    const int cta = (int)blockIdx.x;
    if (cta < pr.ctas0)
        gemv_tma_body<FA, CW, R, 1, 1, false>(smem, sh, cta, pr.ctas0, pr.L[0], pr.w[0], x, pr.y[0], none, 0, pr.P[0],
                                              solo, fu);
    else
        gemv_tma_body<FB, CW, R, 1, 1, false>(smem, sh, cta - pr.ctas0, (int)gridDim.x - pr.ctas0, pr.L[1], pr.w[1],
                                              x, pr.y[1], none, 0, pr.P[1], solo, fu);
}

// ---------------------------------------------- GEMV (resident row range)
//
// Small matrices (the decode step's projections, configuration 0): every CTA
// owns a contiguous row range small enough to sit in shared memory whole
// (of one matrix, or of two matrices that share x -- the decode step's gate
// and up of different formats).  Thread 0 issues the bulk copies of all of
// the CTA's rows on one mbarrier before griddepcontrol.wait.  Exactly two
// such CTAs fit on an SM (each reserves at least kLiteSmemFloor bytes), one
// per SM per launch: under programmatic dependent launch the CTA of the next
// launch of a stream is resident beside the current one and copies its
// weights while the current one computes, so a chain of launches costs about
// one activation hand-off per launch instead of a pipeline fill, and no SM
// ever holds two CTAs of one launch.
constexpr int kLiteWarps = 8;
constexpr uint32_t kLiteRowBudget = 72u * 1024u;   // one CTA's rows of both matrices
constexpr uint32_t kLiteXBudget = 16u * 1024u;     // quantized x (up to 6,553 columns)
constexpr uint32_t kLiteSmemFloor = 77u * 1024u;   // three CTAs never fit in an SM's 228 KB

struct LiteMat {
    Layout L;
    const uint8_t *w;
    float *y;
    const float *add;  // y[row] = (W x)[row] + add[row] when non-null (may alias y)
    uint32_t soff;     // offset of the CTA's rows in the dynamic shared memory
};
struct LitePlan {
    LiteMat m[2];
    int nmat;              // 1 or 2 (two: equal columns and x slice layout)
    uint32_t x_bytes;      // quantized x, rounded to 128
    uint32_t smem;         // dynamic shared memory of a CTA
    unsigned int *status;  // the calling thread's status word, or null
};

__device__ __forceinline__ void lite_rows_of(int rows, int *r0, int *r1)
{
    *r0 = (int)((long long)rows * blockIdx.x / gridDim.x);
    *r1 = (int)((long long)rows * (blockIdx.x + 1) / gridDim.x);
}

// This CTA's rows of one matrix from its shared-memory copy at srow, times
// scale (the RMSNorm prologue's 1 / sqrt(mean(x^2) + eps), else 1), plus the
// epilogue's add.  Row groups of R go to the warps round robin, starting at
// warp `first` (the second matrix of a pair starts where the first one's
// last group went, so their tails land on different warps); lanes stride over
// chunks.
template <uint32_t FMT, int R>
__device__ __forceinline__ unsigned long long lite_rows(const LiteMat &M, uint32_t srow, const XS &s, float scale,
                                                        int first, bool want_key, int index_base)
{
    constexpr int NSL = W<FMT>::kSlices;
    const Layout &L = M.L;
    const int lane = threadIdx.x & 31, C = L.C;
    const int warp = ((threadIdx.x >> 5) + kLiteWarps - first) % kLiteWarps;
    int r0, r1;
    lite_rows_of(L.rows, &r0, &r1);
    const int nr = r1 - r0;
    unsigned long long best = 0ull;
    for (int lr0 = warp * R; lr0 < nr; lr0 += kLiteWarps * R) {
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.f;
        for (int c = lane; c < C; c += 32) {
            W<FMT> wv[R];
#pragma unroll
            for (int i = 0; i < R; ++i)  // rows past the range re-read the last row (in bounds, never written)
                wv[i].load_smem(srow + (uint32_t)min(lr0 + i, nr - 1) * (uint32_t)L.row_stride, L, c);
            const XR<NSL> xr = load_xr<NSL>(s, C, c);
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] += wv[i].dot(xr);
        }
        float out = 0.f;
#pragma unroll
        for (int i = 0; i < R; ++i) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
            if (lane == i) out = acc[i];
        }
        if (lane < R && lr0 + lane < nr) {
            const int row = r0 + lr0 + lane;
            out *= scale;
            if (M.add != nullptr) out += __ldcg(M.add + row);
            M.y[row] = out;
            if (want_key) best = max_ull(best, make_key(out, index_base + row));
        }
    }
    return best;
}

// Warp that takes the row group after matrix M's last one.
__device__ __forceinline__ int lite_next_warp(const LiteMat &M, int R)
{
    int r0, r1;
    lite_rows_of(M.L.rows, &r0, &r1);
    return ((r1 - r0 + R - 1) / R) % kLiteWarps;
}

template <uint32_t FA, uint32_t FB, int R>
__global__ void __launch_bounds__(kLiteWarps * 32, 2)
gemv_lite_kernel(LitePlan P, const float *__restrict__ x, ArgmaxOut am, int want_argmax, Fuse fu)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) unsigned long long bar;
    __shared__ float sumsq[kLiteWarps];
    __shared__ unsigned long long kscratch[kLiteWarps + 1];
    __shared__ int special;
    constexpr int NT = kLiteWarps * 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bar_a = (uint32_t)__cvta_generic_to_shared(&bar);
    const uint32_t rows_a = (uint32_t)__cvta_generic_to_shared(smem + P.x_bytes);
    // The next launch of the stream may start now: it only copies its own
    // weights until its griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        mbar_init(bar_a, 1u);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        special = 0;
        uint32_t total = 0;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (i >= P.nmat) break;
            int r0, r1;
            lite_rows_of(P.m[i].L.rows, &r0, &r1);
            total += (uint32_t)(r1 - r0) * (uint32_t)P.m[i].L.row_stride;
        }
        mbar_expect_tx(bar_a, total);  // with no bytes the arrival alone completes the phase
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (i >= P.nmat) break;
            int r0, r1;
            lite_rows_of(P.m[i].L.rows, &r0, &r1);
            const uint32_t bytes = (uint32_t)(r1 - r0) * (uint32_t)P.m[i].L.row_stride;
            const uint8_t *src = P.m[i].w + (uint64_t)r0 * P.m[i].L.row_stride;
            for (uint32_t off = 0; off < bytes; off += 32768u)
                bulk_g2s(rows_a + P.m[i].soff + off, src + off, min(32768u, bytes - off), bar_a);
        }
        prefetch_share(fu, (int)blockIdx.x, (int)gridDim.x);
    }
    // x (and add) may be written by the previous launch: read through L2
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const Layout &L0 = P.m[0].L;
    // One pass over x: the RMSNorm prologue quantizes x * norm and scales the
    // row sums by 1 / sqrt(mean(x^2) + eps), whose sum of squares is gathered
    // in the same pass.
    const int pre = fu.pre == kPreRmsNorm ? kPreScale : fu.pre;
    const float *aux = fu.pre == kPreRmsNorm ? fu.norm : fu.up;
    float ss = 0.f;
    quantize_x<FA, NT, true>(x, L0.cols, L0.C, smem, 1, 0, pre, 1.f, aux, &special, &ss);
    if (fu.pre == kPreRmsNorm) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
        if (lane == 0) sumsq[warp] = ss;
    }
    __syncthreads();
    float denom = 1.f, scale = 1.f;
    if (fu.pre == kPreRmsNorm) {
        ss = 0.f;
#pragma unroll
        for (int i = 0; i < kLiteWarps; ++i) ss += sumsq[i];
        denom = sqrtf(ss / (float)L0.cols + fu.eps);
        scale = 1.f / denom;
    }
    // every thread waits for the rows (bounded); the phase completes once
    bool landed = mbar_wait(bar_a, 0u);
    if (!__syncthreads_and(landed)) {
        if (tid == 0) {
            report_status(P.status, kStatusConsumerTimeout);
            // copies still in flight must land before the CTA exits
            if (!landed && !mbar_wait(bar_a, 0u)) report_status(P.status, kStatusDrainTimeout);
        }
        return;
    }
    unsigned long long best = 0ull;
    const bool key = want_argmax != 0 && P.nmat == 1;
    if (*(volatile int *)&special != 0) {
        // x holds a NaN/Inf or tiny block: these rows in fp32 from global memory
        const XVal xv{x, fu.pre, denom, aux};
        int r0, r1;
        lite_rows_of(P.m[0].L.rows, &r0, &r1);
        best = fp32_rows<FA>(P.m[0].L, P.m[0].w, r0, r1, warp, kLiteWarps, xv, P.m[0].y, P.m[0].add, key,
                             am.index_base);
        if constexpr (FB != 0) {
            lite_rows_of(P.m[1].L.rows, &r0, &r1);
            fp32_rows<FB>(P.m[1].L, P.m[1].w, r0, r1, warp, kLiteWarps, xv, P.m[1].y, P.m[1].add, false, 0);
        }
    } else {
        const XS s = xs_view(smem, L0.cols);
        best = lite_rows<FA, R>(P.m[0], rows_a + P.m[0].soff, s, scale, 0, key, am.index_base);
        if constexpr (FB != 0)
            lite_rows<FB, R>(P.m[1], rows_a + P.m[1].soff, s, scale, lite_next_warp(P.m[0], R), false, 0);
    }
    if (key) {
        best = block_max_key(best, kscratch);
        finish_argmax(best, am, kscratch);
    }
}

// ------------------------------------ batched projection on int8 tensor cores
//
// Up to 8 positions (the reference's prefill chunk, configuration 3 at
// P = 8) for the 32-weight block formats, on mma.sync m16n8k32 integer tensor
// cores: A = 16 rows x 32 weights of one block (Q8_0 signed, Q5_0 unsigned
// 0..31), B = 32 x values x 8 positions of one plane of the quantized x (hi
// and lo int8 planes, two MMAs), exact int32 sums; each (row, position, block)
// then takes the block's scales exactly as the CUDA-core dot does
// ((d s) (256 hi + lo), Q5_0 minus 16 d s-weighted slice sums).  A CTA's rows
// sit in shared memory whole (bulk copies before griddepcontrol.wait, as the
// resident-row-range GEMV); warp w takes blocks [w C / 8, (w + 1) C / 8) of
// every 16-row tile, and the warps' partial tiles are added in warp order.
// A special x computes every position's rows in fp32.
constexpr int kMmaWarps = 8;
constexpr int kMmaMaxTiles = 4;  // 64 rows per CTA

template <uint32_t FMT>
__device__ __forceinline__ void mma_blk(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    if constexpr (FMT == kQ8_0)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Weights k = 4t..4t+3 (lo) and 16+4t..16+4t+3 (hi) of block c of the row
// staged at srow, as A-fragment words; *d the block's scale.
template <uint32_t FMT>
__device__ __forceinline__ void mma_row_words(uint32_t srow, const Layout &L, int c, int t, uint32_t *lo,
                                              uint32_t *hi, float *d)
{
    if constexpr (FMT == kQ8_0) {
        *lo = lds32(srow + (uint32_t)(c << 4) + 4u * t);
        *hi = lds32(srow + (uint32_t)((L.C + c) << 4) + 4u * t);
        *d = f16_fast(lds16(srow + L.off_a + 2u * c));
    } else {
        // byte i of qs: weight i (low nibble), weight i + 16 (high nibble);
        // bit i of qh: the fifth bit of weight i
        const uint32_t q = lds32(srow + (uint32_t)(c << 4) + 4u * t);
        const uint32_t qh = lds32(srow + L.off_a + 4u * c);
        *lo = (q & 0x0f0f0f0fu) | spread4(qh >> (4 * t));
        *hi = ((q >> 4) & 0x0f0f0f0fu) | spread4(qh >> (16 + 4 * t));
        *d = f16_fast(lds16(srow + L.off_b + 2u * c));
    }
}

template <uint32_t FMT>
__global__ void __launch_bounds__(kMmaWarps * 32, 1)
matmul_mma_kernel(Layout L, const uint8_t *__restrict__ w, const float *__restrict__ X, int np, float *__restrict__ Y,
                  uint32_t x_bytes, unsigned int *status)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) unsigned long long bar;
    __shared__ int special;
    __shared__ float part[kMmaWarps][kMmaMaxTiles][16 * 8];
    constexpr int NT = kMmaWarps * 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t bar_a = (uint32_t)__cvta_generic_to_shared(&bar);
    const uint32_t rows_a = (uint32_t)__cvta_generic_to_shared(smem + x_bytes);
    const int r0 = (int)((long long)L.rows * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)L.rows * (blockIdx.x + 1) / gridDim.x);
    const int nr = r1 - r0, ntiles = (nr + 15) / 16;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (tid == 0) {
        mbar_init(bar_a, 1u);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        special = 0;
        const uint32_t bytes = (uint32_t)nr * (uint32_t)L.row_stride;
        mbar_expect_tx(bar_a, bytes);
        const uint8_t *src = w + (uint64_t)r0 * L.row_stride;
        for (uint32_t off = 0; off < bytes; off += 32768u)
            bulk_g2s(rows_a + off, src + off, min(32768u, bytes - off), bar_a);
    }
    // X may be written by the previous launch: read through L2
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t xb = xs_bytes(L.cols);
    quantize_x<FMT, NT, true>(X, L.cols, L.C, smem, np, xb, kPreNone, 1.f, nullptr, &special);
    __syncthreads();
    const bool landed = mbar_wait(bar_a, 0u);
    if (!__syncthreads_and(landed)) {
        if (tid == 0) {
            report_status(status, kStatusConsumerTimeout);
            if (!landed && !mbar_wait(bar_a, 0u)) report_status(status, kStatusDrainTimeout);
        }
        return;
    }
    if (*(volatile int *)&special != 0) {
        for (int p = 0; p < np; ++p)
            fp32_rows<FMT>(L, w, r0, r1, warp, kMmaWarps, XVal{X + (size_t)p * L.cols, kPreNone, 1.f, nullptr},
                           Y + (size_t)p * L.rows, nullptr, false, 0);
        return;
    }
    const int C = L.C;
    const int k0 = C * warp / kMmaWarps, k1 = C * (warp + 1) / kMmaWarps;
    float acc[kMmaMaxTiles][4];
#pragma unroll
    for (int ti = 0; ti < kMmaMaxTiles; ++ti) {
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[ti][j] = 0.f;
    }
    // B column g: position g (positions past np re-read the last one, never written)
    const uint32_t xh = (uint32_t)__cvta_generic_to_shared(smem + (size_t)min(g, np - 1) * xb);
    const uint32_t xl = xh + (uint32_t)L.cols;
    // C columns 2t, 2t + 1: the scales of those positions' slices
    const float2 *reca = reinterpret_cast<const float2 *>(smem + (size_t)min(2 * t, np - 1) * xb + 2 * (size_t)L.cols);
    const float2 *recb =
        reinterpret_cast<const float2 *>(smem + (size_t)min(2 * t + 1, np - 1) * xb + 2 * (size_t)L.cols);
    for (int c = k0; c < k1; ++c) {
        const uint32_t bh0 = lds32(xh + (uint32_t)(c << 4) + 4u * t);
        const uint32_t bh1 = lds32(xh + (uint32_t)((C + c) << 4) + 4u * t);
        const uint32_t bl0 = lds32(xl + (uint32_t)(c << 4) + 4u * t);
        const uint32_t bl1 = lds32(xl + (uint32_t)((C + c) << 4) + 4u * t);
        const float2 sa = reca[c], sb = recb[c];
        float ma = 0.f, mb = 0.f;  // Q5_0: 16 (s sum of slice c + s sum of slice C + c)
        if constexpr (FMT == kQ5_0) {
            ma = 16.f * (sa.y + reca[C + c].y);
            mb = 16.f * (sb.y + recb[C + c].y);
        }
#pragma unroll
        for (int ti = 0; ti < kMmaMaxTiles; ++ti) {
            if (ti >= ntiles) break;  // uniform over the warp
            const int ra = min(ti * 16 + g, nr - 1), rb = min(ti * 16 + g + 8, nr - 1);
            uint32_t a[4];
            float da, db;
            mma_row_words<FMT>(rows_a + (uint32_t)ra * (uint32_t)L.row_stride, L, c, t, &a[0], &a[2], &da);
            mma_row_words<FMT>(rows_a + (uint32_t)rb * (uint32_t)L.row_stride, L, c, t, &a[1], &a[3], &db);
            int dh[4] = {0, 0, 0, 0}, dl[4] = {0, 0, 0, 0};
            mma_blk<FMT>(dh, a, bh0, bh1);
            mma_blk<FMT>(dl, a, bl0, bl1);
            // D: (ra, 2t), (ra, 2t + 1), (rb, 2t), (rb, 2t + 1); the block's
            // scales in the order of the CUDA-core dot (W<FMT>::dot_u)
            if constexpr (FMT == kQ8_0) {
                acc[ti][0] += (da * sa.x) * (float)(dh[0] * 256 + dl[0]);
                acc[ti][1] += (da * sb.x) * (float)(dh[1] * 256 + dl[1]);
                acc[ti][2] += (db * sa.x) * (float)(dh[2] * 256 + dl[2]);
                acc[ti][3] += (db * sb.x) * (float)(dh[3] * 256 + dl[3]);
            } else {
                acc[ti][0] += da * (sa.x * (float)(dh[0] * 256 + dl[0]) - ma);
                acc[ti][1] += da * (sb.x * (float)(dh[1] * 256 + dl[1]) - mb);
                acc[ti][2] += db * (sa.x * (float)(dh[2] * 256 + dl[2]) - ma);
                acc[ti][3] += db * (sb.x * (float)(dh[3] * 256 + dl[3]) - mb);
            }
        }
    }
#pragma unroll
    for (int ti = 0; ti < kMmaMaxTiles; ++ti) {
        if (ti >= ntiles) break;
        part[warp][ti][g * 8 + 2 * t] = acc[ti][0];
        part[warp][ti][g * 8 + 2 * t + 1] = acc[ti][1];
        part[warp][ti][(g + 8) * 8 + 2 * t] = acc[ti][2];
        part[warp][ti][(g + 8) * 8 + 2 * t + 1] = acc[ti][3];
    }
    __syncthreads();
    // the warps' K ranges added in warp order
    for (int e = tid; e < ntiles * 128; e += NT) {
        const int ti = e >> 7, rr = (e >> 3) & 15, n = e & 7, row = ti * 16 + rr;
        if (row < nr && n < np) {
            float v = part[0][ti][rr * 8 + n];
#pragma unroll
            for (int q = 1; q < kMmaWarps; ++q) v += part[q][ti][rr * 8 + n];
            Y[(size_t)n * L.rows + r0 + row] = v;
        }
    }
}

// ------------------------------------------------------------- matmul
//
// Batched form for up to NP positions per launch (the reference's chunk of
// 8 positions).  quantize_x_kernel writes the quantized x of every position
// once, as the shared-memory image the GEMV kernels build (hi | lo |
// records, xs_bytes(cols) per position), and every matmul CTA copies that
// image into shared memory.  The matmul kernel is launched with programmatic
// dependent launch: its first weight loads are issued before
// griddepcontrol.wait, so they overlap the quantization kernel.  Groups of
// TPT lanes take rows with the same one-deep prefetch over (row, chunk)
// items as gemv_kernel; each loaded chunk is unpacked once and applied to
// every position.

template <uint32_t FMT>
__global__ void __launch_bounds__(kThreads)
quantize_x_kernel(const float *__restrict__ X, int cols, int C, uint8_t *__restrict__ xq, size_t xb)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    quantize_x<FMT>(X + (size_t)blockIdx.x * cols, cols, C, xq + (size_t)blockIdx.x * xb);
}

template <uint32_t FMT, int TPT, int NP>
__global__ void __launch_bounds__(kThreads)
matmul_kernel(Layout L, const uint8_t *__restrict__ w, const uint8_t *__restrict__ xq, int np,
              float *__restrict__ Y)
{
    static_assert(TPT >= NP, "lane p of a row group writes position p");
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NSL = W<FMT>::kSlices;
    const int C = L.C;
    const size_t xb = xs_bytes(L.cols);
    constexpr int GPW = 32 / TPT;
    const int lane = threadIdx.x & 31;
    const int grp = lane / TPT, gl = lane % TPT;
    const int wg = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    const int wtot = gridDim.x * (kThreads / 32);
    const int NI = (C + TPT - 1) / TPT;
    const int tiles = (L.rows + GPW - 1) / GPW;
    const int my_tiles = wg < tiles ? (tiles - 1 - wg) / wtot + 1 : 0;
    const int n_items = my_tiles * NI;

    // Item k = (tile t, chunk iteration it); both advance incrementally.
    auto load_item = [&](int t, int it, W<FMT> &dst) {
        const int c = it * TPT + gl, row = t * GPW + grp;
        if (c < C && row < L.rows)
            dst.load(w + (uint64_t)row * L.row_stride, L, c);
        else
            dst.zero();
    };
    W<FMT> bufa, bufb;
    int t = wg, it = 0;
    if (n_items > 0) load_item(t, it, bufa);

    // x comes from quantize_x_kernel, the launch this one depends on
    asm volatile("griddepcontrol.wait;" ::: "memory");
    {
        const uint4 *src = reinterpret_cast<const uint4 *>(xq);
        uint4 *dst = reinterpret_cast<uint4 *>(smem);
        const int n16 = (int)((size_t)np * xb / 16);
        for (int i = threadIdx.x; i < n16; i += kThreads) dst[i] = src[i];
    }
    __syncthreads();

    float acc[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p] = 0.f;
    // Compute item (t, it) from `use` while `pre` receives item k+1.
    auto step = [&](int k, int &t, int &it, W<FMT> &use, W<FMT> &pre) {
        int nt = t, nit = it + 1;
        if (nit == NI) {
            nit = 0;
            nt += wtot;
        }
        if (k + 1 < n_items) load_item(nt, nit, pre);
        const int c = it * TPT + gl;
        if (c < C) {
            const typename W<FMT>::U u = use.unpack();
#pragma unroll
            for (int p = 0; p < NP; ++p)
                if (p < np) acc[p] += W<FMT>::dot_u(u, load_xr<NSL>(xs_view(smem + p * xb, L.cols), C, c));
        }
        if (it == NI - 1) {
#pragma unroll
            for (int p = 0; p < NP; ++p) {
#pragma unroll
                for (int o = TPT / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(kFull, acc[p], o);
            }
            float out = 0.f;
#pragma unroll
            for (int p = 0; p < NP; ++p)
                if (gl == p) out = acc[p];
            const int row = t * GPW + grp;
            if (gl < np && row < L.rows) Y[(size_t)gl * L.rows + row] = out;
#pragma unroll
            for (int p = 0; p < NP; ++p) acc[p] = 0.f;
        }
        t = nt;
        it = nit;
    };
    for (int k = 0; k < n_items; k += 2) {
        step(k, t, it, bufa, bufb);
        if (k + 1 < n_items) step(k + 1, t, it, bufb, bufa);
    }
}

// ---------------------------------------------- matmul (tensor cores)
//
// Batched projection of many positions on the 5th-generation tensor cores
// (src/quantized_matvec.cpp:164-224 computes the same Y[p] = W X[p]).
// Operands are split into bf16 pairs, w = wh + wl and x = xh + xl, and each
// 16-wide K slice issues wh*xh + wl*xh + wh*xl as tcgen05.mma (kind::f16,
// bf16 inputs, fp32 accumulator in tensor memory).  wl and xl carry the next
// 8 bits, so every product is exact to about 2^-16 of |w x|, far inside the
// parity bound 1e-4 * sum|w x|.
//
//  * split_x_kernel (once per call) writes x of every position tile as
//    stage images: for each 32-wide K step the xh and xl planes of TN
//    positions in the canonical K-major no-swizzle layout (8-row x 16-byte
//    core matrices; 16-byte unit u of a plane at byte u * 16), so a stage is
//    one contiguous bulk copy.  A word per position tile flags any x outside
//    the range the split handles.
//  * matmul_tc_kernel: a CTA owns 128 rows x TN positions.  Thread 0 keeps
//    the x planes of the next stages in flight with cp.async.bulk (no
//    multicast), completing on one mbarrier per stage.  All 512 threads
//    decode the stage's 128 x 32 weights from the resident layout to the
//    reference's fp32 values (raw bytes prefetched into registers a stage
//    ahead), split them and store the planes; thread 0 then waits for the
//    stage's x, issues its 6 MMAs and commits them to the mbarrier that frees
//    the stage.  The epilogue reads the accumulator with tcgen05.ld (warp w
//    reads lanes 32 (w % 4) .. + 31) and writes Y[p][row], one 128-byte run
//    per warp store.
//
// A tile that holds a non-finite weight scale, or an x outside the split's
// range, is recomputed on the CUDA cores in fp32 so that Inf and NaN
// propagate as in the reference's loop; the split planes could otherwise
// turn Inf * 0 into NaN.

constexpr int kTcM = 128;         // rows per tile = accumulator lanes
constexpr int kTcK = 64;          // K per stage
constexpr int kTcThreads = 512;   // weight-decode threads (16 warps)
constexpr uint32_t kTcSmemBudget = 220u * 1024u;
constexpr uint32_t kTcACol = 256u;  // weight ring after the 256 accumulator columns
constexpr int kTcMaxStages = (512 - (int)kTcACol) / kTcK;  // a stage: wh | wl, kTcK / 2 columns each
constexpr int kTcUnits = kTcK / 32;  // 8-weight units per decode thread and stage
constexpr unsigned int kStatusMmaTimeout = 16u;

// Shared memory of one stage: xh | xl (TN x kTcK bf16 each).  The weights of
// a stage (wh | wl, kTcK / 2 columns each) live in tensor memory.
__host__ __device__ constexpr uint32_t tc_plane_x(int tn) { return (uint32_t)tn * kTcK * 2u; }
__host__ __device__ constexpr uint32_t tc_stage_bytes(int tn) { return 2u * tc_plane_x(tn); }

// Stages that fit the shared-memory budget (at most kTcMaxStages).
__host__ __device__ constexpr int tc_stages(int tn)
{
    return kTcSmemBudget / tc_stage_bytes(tn) > (uint32_t)kTcMaxStages ? kTcMaxStages
                                                                      : (int)(kTcSmemBudget / tc_stage_bytes(tn));
}

// Split-x scratch: the stage images, position tile-major.
// 2^23 + (byte I of w), exactly: the byte becomes the low mantissa bits of a
// float whose exponent is that of 2^23.  Integer-to-float without the
// conversion pipe; callers subtract 2^23 (plus any offset) exactly.
template <int I>
__device__ __forceinline__ float u8_magic(uint32_t w)
{
    return __uint_as_float(__byte_perm(w, 0x4b000000u, 0x7540u | I));
}

// Packed two-wide fp32 arithmetic (one instruction for both lanes of a
// float2, each rounded exactly as the scalar operation).
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// v[4 j + i] = (2^23 + byte i of n[j]) - bias, exact for bias = 2^23 + offset
__device__ __forceinline__ void bytes_to_float(uint32_t n0, uint32_t n1, float bias, float v[8])
{
    const float2 nb = f2(-bias, -bias);
    const float2 a = __fadd2_rn(f2(u8_magic<0>(n0), u8_magic<1>(n0)), nb);
    const float2 b = __fadd2_rn(f2(u8_magic<2>(n0), u8_magic<3>(n0)), nb);
    const float2 c = __fadd2_rn(f2(u8_magic<0>(n1), u8_magic<1>(n1)), nb);
    const float2 d = __fadd2_rn(f2(u8_magic<2>(n1), u8_magic<3>(n1)), nb);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

// v[i] *= s, rounded once per element
__device__ __forceinline__ void scale8(float s, float v[8])
{
    const float2 s2 = f2(s, s);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 r = __fmul2_rn(f2(v[2 * j], v[2 * j + 1]), s2);
        v[2 * j] = r.x;
        v[2 * j + 1] = r.y;
    }
}

// Raw bytes of 8 consecutive weights (k0 .. k0 + 7, k0 a multiple of 8) of
// one resident row, and their decoding to fp32 with the reference's
// arithmetic (src/quantization.cpp:54-67, 161-184, 380-409, 588-615): every
// product below is exact or rounds once, as there.
// Loads of the raw bytes: read-only global loads, or plain loads when the
// tile's rows have been copied to shared memory (same offsets).
template <bool SMEM, typename T>
__device__ __forceinline__ T ld_raw(const uint8_t *p)
{
    if constexpr (SMEM) return *(const T *)p;
    else return __ldg((const T *)p);
}

template <uint32_t FMT> struct Raw8;

template <> struct Raw8<kQ8_0> {
    static constexpr bool kExactLo = false;
    uint2 q;
    uint32_t d;
    template <bool SMEM = false>
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int k0)
    {
        const int b = k0 >> 5, i0 = k0 & 31;
        q = ld_raw<SMEM, uint2>(row + (((i0 < 16) ? b : L.C + b) << 4) + (i0 & 8));
        d = ld_raw<SMEM, unsigned short>(row + L.off_a + 2 * b);
    }
    __device__ __forceinline__ bool decode(int, float v[8]) const
    {
        // signed bytes biased by 128 so that they read as unsigned
        bytes_to_float(q.x ^ 0x80808080u, q.y ^ 0x80808080u, 8388736.0f, v);
        scale8(f16_fast(d), v);
        return (d & 0x7c00u) != 0x7c00u;
    }
};

template <> struct Raw8<kQ5_0> {
    // d (11 significant bits) times an integer in [-16, 15]: at most 16
    // significant bits, so w - round8(w) is already an exact bf16
    static constexpr bool kExactLo = true;
    uint2 q;
    uint32_t qh, d;
    template <bool SMEM = false>
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int k0)
    {
        const int b = k0 >> 5, i0 = k0 & 31;
        q = ld_raw<SMEM, uint2>(row + (b << 4) + (i0 & 8));
        qh = ld_raw<SMEM, uint32_t>(row + L.off_a + 4 * b) >> i0;
        d = ld_raw<SMEM, unsigned short>(row + L.off_b + 2 * b);
    }
    __device__ __forceinline__ bool decode(int k0, float v[8]) const
    {
        // weight i of the block: low nibble of byte i (i < 16) or high nibble
        // of byte i - 16, fifth bit = bit i of qh; value (n - 16) * d
        const int sh = (k0 & 16) ? 4 : 0;
        const uint32_t n0 = ((q.x >> sh) & 0x0f0f0f0fu) | spread4(qh);
        const uint32_t n1 = ((q.y >> sh) & 0x0f0f0f0fu) | spread4(qh >> 4);
        bytes_to_float(n0, n1, 8388624.0f, v);
        scale8(f16_fast(d), v);
        return (d & 0x7c00u) != 0x7c00u;
    }
};

template <> struct Raw8<kQ4_K> {
    static constexpr bool kExactLo = false;
    uint2 q;
    uint4 hdr;
    template <bool SMEM = false>
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int k0)
    {
        const int sb = k0 >> 8, j = (k0 >> 5) & 7, o0 = k0 & 31;
        const int c = 4 * sb + (j >> 1);
        q = ld_raw<SMEM, uint2>(row + (((o0 < 16) ? c : L.C + c) << 4) + (o0 & 8));
        hdr = ld_raw<SMEM, uint4>(row + L.off_a + (sb << 4));
    }
    __device__ __forceinline__ bool decode(int k0, float v[8]) const
    {
        // 6-bit scale and minimum of sub-block j (src/quantization.cpp:351-378);
        // header bytes 4..15 are the 12 packed scale bytes
        const int j = (k0 >> 5) & 7, t = 8 * (j & 3);
        uint32_t sc, mn;
        if (j < 4) {
            sc = (hdr.y >> t) & 63u;
            mn = (hdr.z >> t) & 63u;
        } else {
            sc = ((hdr.w >> t) & 15u) | (((hdr.y >> t) >> 6 & 3u) << 4);
            mn = ((hdr.w >> t) >> 4 & 15u) | (((hdr.z >> t) >> 6 & 3u) << 4);
        }
        const float scale = __fmul_rn(f16_fast(hdr.x & 0xffffu), (float)sc);
        const float minimum = __fmul_rn(f16_fast(hdr.x >> 16), (float)mn);
        const int sh = 4 * (j & 1);
        bytes_to_float((q.x >> sh) & 0x0f0f0f0fu, (q.y >> sh) & 0x0f0f0f0fu, 8388608.0f, v);
        // scale * q is exact, so one fused rounding equals the reference's
        // multiply-then-subtract
        const float2 sc2 = f2(scale, scale), mn2 = f2(-minimum, -minimum);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 r = __ffma2_rn(f2(v[2 * j], v[2 * j + 1]), sc2, mn2);
            v[2 * j] = r.x;
            v[2 * j + 1] = r.y;
        }
        return (hdr.x & 0x7c00u) != 0x7c00u && (hdr.x & 0x7c000000u) != 0x7c000000u;
    }
};

template <> struct Raw8<kQ6_K> {
    static constexpr bool kExactLo = false;
    uint2 ql, qh;
    uint32_t sc, d;
    template <bool SMEM = false>
    __device__ __forceinline__ void load(const uint8_t *row, const Layout &L, int k0)
    {
        // weight 128 g + 32 r + o of the super-block lives in chunk
        // 4 sb + 2 g + (o >> 4)
        const int sb = k0 >> 8, g = (k0 >> 7) & 1, r = (k0 >> 5) & 3, o0 = k0 & 31;
        const int c = 4 * sb + 2 * g + (o0 >> 4);
        ql = ld_raw<SMEM, uint2>(row + ((((r & 1) ? L.C : 0) + c) << 4) + (o0 & 8));
        qh = ld_raw<SMEM, uint2>(row + ((2 * L.C + c) << 4) + (o0 & 8));
        sc = ld_raw<SMEM, uint32_t>(row + L.off_a + 4 * c);
        d = ld_raw<SMEM, unsigned short>(row + L.off_b + 2 * sb);
    }
    __device__ __forceinline__ bool decode(int k0, float v[8]) const
    {
        const int r = (k0 >> 5) & 3;
        const int s = (int)(int8_t)((sc >> (8 * r)) & 0xffu);
        const float ds = __fmul_rn(f16_fast(d), (float)s);
        const int shl = 4 * (r >> 1), shh = 2 * r;
        const uint32_t n0 = ((ql.x >> shl) & 0x0f0f0f0fu) | (((qh.x >> shh) & 0x03030303u) << 4);
        const uint32_t n1 = ((ql.y >> shl) & 0x0f0f0f0fu) | (((qh.y >> shh) & 0x03030303u) << 4);
        bytes_to_float(n0, n1, 8388640.0f, v);  // n - 32
        scale8(ds, v);
        return (d & 0x7c00u) != 0x7c00u;
    }
};

// x rounded to 8 significant bits (nearest), as fp32s whose low 16 bits
// are zero, i.e. an exact bf16: Veltkamp's splitting with 2^16 + 1.  The
// explicitly rounded operations keep the compiler from contracting them.
__device__ __forceinline__ float2 round8x2(float2 x)
{
    const float2 m1 = f2(-1.f, -1.f);
    const float2 t = __fmul2_rn(x, f2(65537.0f, 65537.0f));
    return __ffma2_rn(__ffma2_rn(x, m1, t), m1, t);  // t - (t - x)
}

// Split 8 floats into bf16 high and low parts, v = hi + lo + e with
// |hi - v| <= 2^-8 |v| and |e| <= 2^-16 |v|, as packed words (hi[j], lo[j]
// hold elements 2j and 2j + 1, the even one in the low half).  FMA-pipe
// arithmetic and byte permutes only.  |v| must stay below 2^111 (65537 v
// finite).  EXACT_LO: every v has at most 16 significant bits, so v - hi is
// an exact bf16 (e = 0) and needs no rounding.
template <bool EXACT_LO = false>
__device__ __forceinline__ void split_words(const float v[8], uint32_t h[4], uint32_t l[4])
{
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 x = f2(v[2 * j], v[2 * j + 1]);
        const float2 hi = round8x2(x);
        float2 lo = __ffma2_rn(hi, f2(-1.f, -1.f), x);  // x - hi, exact
        if (!EXACT_LO) lo = round8x2(lo);
        h[j] = __byte_perm(__float_as_uint(hi.x), __float_as_uint(hi.y), 0x7632u);
        l[j] = __byte_perm(__float_as_uint(lo.x), __float_as_uint(lo.y), 0x7632u);
    }
}

// The split stored as two 16-byte units (element 0 at the lowest address).
__device__ __forceinline__ void split_store(const float v[8], uint8_t *hi_plane, uint8_t *lo_plane, uint32_t off)
{
    uint32_t h[4], l[4];
    split_words(v, h, l);
    *(uint4 *)(hi_plane + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *(uint4 *)(lo_plane + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices along
// K 128 bytes apart (leading byte offset), 8-row groups kTcK * 16 bytes apart
// (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)(128u >> 4) << 16) |
           ((uint64_t)((kTcK * 16u) >> 4) << 32) | (1ull << 46);
}

// Instruction descriptor: fp32 accumulator, bf16 A and B, both K-major,
// N = tn, M = 128.
__host__ __device__ constexpr uint32_t umma_idesc(int tn)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(tn >> 3) << 17) | ((uint32_t)(kTcM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// Same, with A (128 x 16 bf16: lane = row, two K values per 32-bit column,
// the even one in the low half) read from tensor memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

// 4 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d)
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}

// 8 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t r[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive fp32 accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8])
{
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// x of position pos, column k: X[pos][k], or up[pos][k] * silu(X[pos][k])
// when the source carries the SwiGLU of a [gate | up] pair
// (transformer_swiglu_f32, src/transformer_ops.cpp:163-178).
__device__ __forceinline__ float x_at(const XSource &src, int pos, int k)
{
    const float g = src.x[(size_t)pos * src.ldx + k];
    return src.up ? src.up[(size_t)pos * src.ldu + k] * (g / (1.0f + expf(-g))) : g;
}

// fp32 recomputation of one tile (rows r0.., positions p0..) over columns
// [kb, ke) on the CUDA cores.
template <uint32_t FMT>
__device__ void tc_tile_fallback(const Layout &L, const uint8_t *__restrict__ w, const XSource &src, int np,
                                 float *__restrict__ Y, int r0, int p0, int tn, int kb, int ke)
{
    for (int o = threadIdx.x; o < kTcM * tn; o += blockDim.x) {
        const int row = r0 + (o % kTcM), pos = p0 + (o / kTcM);
        if (row >= L.rows || pos >= np) continue;
        const uint8_t *rp = w + (uint64_t)row * L.row_stride;
        float acc = 0.f;
        for (int k0 = kb; k0 < ke; k0 += 8) {
            Raw8<FMT> raw;
            raw.load(rp, L, k0);
            float v[8];
            raw.decode(k0, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc += v[i] * x_at(src, pos, k0 + i);
        }
        Y[(size_t)pos * L.rows + row] = acc;
    }
}

// x of every position tile -> bf16 stage images (see above).  An x the split
// cannot represent (non-finite, or |x| >= 2^111) becomes NaN in the planes,
// so the tile's accumulator turns non-finite and the tile is recomputed.
template <int TN>
__global__ void __launch_bounds__(kThreads)
split_x_kernel(XSource src, int np, int cols, int nk, uint8_t *__restrict__ xs)
{
    constexpr uint32_t kPlaneX = tc_plane_x(TN);
    constexpr int kUnits = TN * (kTcK / 8);
    // the matmul launched after this kernel may start its weight work now;
    // it reads these images only after its griddepcontrol.wait
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int n_pt = (np + TN - 1) / TN;
    const long long total = (long long)n_pt * nk * kUnits;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
         id += (long long)gridDim.x * blockDim.x) {
        const int u = (int)(id % kUnits);
        const long long img = id / kUnits;  // pt * nk + kc
        const int kc = (int)(img % nk), pt = (int)(img / nk);
        constexpr int KG = kTcK / 8;  // 8-wide K groups per stage
        const int pos = pt * TN + (u / (8 * KG)) * 8 + (u & 7);
        const int k0 = kc * kTcK + ((u >> 3) % KG) * 8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (pos < np && k0 < cols) {
            const float *xp = src.x + (size_t)pos * src.ldx + k0;
            const float4 a = __ldg((const float4 *)xp);
            const float4 b = __ldg((const float4 *)(xp + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            if (src.up) {  // x = up * silu(gate)
                const float *up = src.up + (size_t)pos * src.ldu + k0;
                const float4 c = __ldg((const float4 *)up);
                const float4 d = __ldg((const float4 *)(up + 4));
                const float u[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = u[i] * (v[i] / (1.0f + expf(-v[i])));
            }
        }
        uint8_t *dst = xs + (size_t)img * 2u * kPlaneX;
        split_store(v, dst, dst + kPlaneX, (uint32_t)u * 16u);
    }
}

// WSMEM: the tile's resident rows are copied to shared memory once (when
// they fit) and decoded from there; otherwise each decode thread loads its
// bytes from global memory one stage ahead.  S: x stages in the ring.
// Split K (gridDim.z > 1): CTA z takes stages [z nk / Z, (z + 1) nk / Z) and
// writes its partial products to slice z of Y (np x rows floats each).
template <uint32_t FMT, int TN, bool WSMEM>
__global__ void __launch_bounds__(kTcThreads + 64, 1)
matmul_tc_kernel(Layout L, const uint8_t *__restrict__ w, XSource X, const uint8_t *__restrict__ xs, int np,
                 float *__restrict__ Y, int S, unsigned int *call_status)
{
    static_assert(TN % 16 == 0 && TN >= 32 && TN <= 256, "N of one MMA: a multiple of 16 in 32..256");
    static_assert(kTcM * (kTcK / 8) == kTcThreads * kTcUnits, "kTcUnits weight units per decode thread and stage");
    static_assert(kTcACol + (uint32_t)kTcK * kTcMaxStages <= 512u, "A ring must fit tensor memory");
    // warps 0..15 decode weights, warp 16 issues MMAs, warp 17 copies x
    constexpr int kDecodeWarps = kTcThreads / 32, kMmaWarp = kDecodeWarps, kCopyWarp = kDecodeWarps + 1;
    constexpr uint32_t kPlaneX = tc_plane_x(TN);
    constexpr uint32_t kStage = tc_stage_bytes(TN);
    constexpr uint32_t kIdesc = umma_idesc(TN);

    extern __shared__ __align__(128) uint8_t smem[];
    // [0, S) weights stored, [S, 2S) x landed, [2S, 3S) MMAs done, then the
    // weight tile's arrival
    __shared__ __align__(8) unsigned long long bars[3 * kTcMaxStages + 1];
    __shared__ uint32_t tmem_slot;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = blockIdx.x * kTcM, pt = blockIdx.y, p0 = pt * TN;
    const int nk = (L.cols + kTcK - 1) / kTcK;
    const int kc0 = (int)((long long)nk * blockIdx.z / gridDim.z), kc1 = (int)((long long)nk * (blockIdx.z + 1) / gridDim.z);
    const int nloc = kc1 - kc0;  // this CTA's stages (>= 1: the host keeps splits <= nk)
    Y += (size_t)blockIdx.z * (size_t)np * (size_t)L.rows;
    const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t wbar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]);
    const uint32_t xbar0 = wbar0 + 8u * S, ebar0 = wbar0 + 16u * S, tbar = wbar0 + 24u * S;
    const int tile_rows = L.rows - r0 < kTcM ? L.rows - r0 : kTcM;
    const uint32_t tile_bytes = (uint32_t)tile_rows * (uint32_t)L.row_stride;
    const uint8_t *wtile = smem + (size_t)S * kStage;  // WSMEM: resident rows r0 .. r0 + tile_rows

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(wbar0 + 8u * i, (uint32_t)kDecodeWarps);
            mbar_init(xbar0 + 8u * i, 1u);
            mbar_init(ebar0 + 8u * i, 1u);
        }
        mbar_init(tbar, 1u);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        // all 512 columns: accumulator in [0, TN), weight stages from kTcACol
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(&tmem_slot)),
                     "r"(512u));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    bool ok = true;
    int issued = 0;  // x copies issued (copy thread)
    if (warp == kCopyWarp) {
        // ------------------------------------------------ x stage copies
        if (lane == 0) {
            if (WSMEM) {
                // the tile's rows are contiguous: one run of tile_bytes
                mbar_expect_tx(tbar, tile_bytes);
                const uint8_t *src = w + (uint64_t)r0 * L.row_stride;
                const uint32_t dst = smem0 + (uint32_t)S * kStage;
                for (uint32_t off = 0; off < tile_bytes; off += 32768u)
                    bulk_g2s(dst + off, src + off, min(32768u, tile_bytes - off), tbar);
            }
            const uint8_t *ximg = xs + (size_t)pt * nk * (size_t)kStage;
            // the x images come from split_x_kernel, the launch this one
            // depends on (programmatic dependent launch)
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int j = 0; j < nloc; ++j) {
                const int s = j % S;
                // buffer s is free once the MMAs of stage j - S are done
                if (j >= S && !mbar_wait_idle(ebar0 + 8u * s, (uint32_t)((j / S - 1) & 1))) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(xbar0 + 8u * s, kStage);
                bulk_g2s(smem0 + (uint32_t)s * kStage, ximg + (size_t)(kc0 + j) * kStage, kStage, xbar0 + 8u * s);
                issued = j + 1;
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------ MMA issue
        if (lane == 0) {
            for (int kc = 0; kc < nloc; ++kc) {  // local stage index
                const int s = kc % S;
                const uint32_t par = (uint32_t)((kc / S) & 1);
                if (!mbar_wait_idle(wbar0 + 8u * s, par) || !mbar_wait_idle(xbar0 + 8u * s, par)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_h = tmem + kTcACol + (uint32_t)kTcK * s, a_l = a_h + kTcK / 2;
                const uint32_t b_h = smem0 + (uint32_t)s * kStage, b_l = b_h + kPlaneX;
#pragma unroll
                for (int j = 0; j < kTcK / 16; ++j) {
                    // K slice j: 8 columns of A, two core matrices along K of B
                    umma_bf16_ts(tmem, a_h + 8u * j, umma_desc(b_h + 256u * j), kIdesc, (kc | j) != 0);
                    umma_bf16_ts(tmem, a_l + 8u * j, umma_desc(b_h + 256u * j), kIdesc, 1u);
                    umma_bf16_ts(tmem, a_h + 8u * j, umma_desc(b_l + 256u * j), kIdesc, 1u);
                }
                umma_commit(ebar0 + 8u * s);
            }
        }
    } else {
        // ------------------------------------------------ weight decode
        // Warp w owns tensor-memory lanes 32 (w % 4) .. + 31 (tile rows) and
        // K range w / 4 of every stage: kTcUnits 8-weight units, 4 columns
        // each per plane.  A stage's stores are published (wait::st, then the
        // arrival) only after the next stage has been decoded, so their
        // latency overlaps that work.
        const int q = warp & 3, kp = warp >> 2;
        const int wrow_i = r0 + 32 * q + lane;
        const bool have_row = wrow_i < L.rows;
        const uint8_t *wrow = WSMEM ? wtile + (size_t)(32 * q + lane) * L.row_stride
                                    : w + (uint64_t)(have_row ? wrow_i : 0) * L.row_stride;
        const int wk = kc0 * kTcK + kp * 8 * kTcUnits;  // first column of this thread's range
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + kTcACol + 4u * kTcUnits * kp;
        if (WSMEM && !mbar_wait(tbar, 0u)) ok = false;
        Raw8<FMT> wr[kTcUnits];
        if (!WSMEM) {
#pragma unroll
            for (int u = 0; u < kTcUnits; ++u)
                if (have_row && wk + 8 * u < L.cols) wr[u].load(wrow, L, wk + 8 * u);
        }
        int pending = -1;  // buffer whose tensor-memory stores are not yet published
        int s = 0, round = 0;  // buffer and ring round of stage kc
        for (int kc = 0; kc < nloc; ++kc, s = (s + 1 == S ? 0 : s + 1), round += (s == 0)) {
            const int k0 = kc * kTcK + wk;
            Raw8<FMT> wn[kTcUnits];
            uint32_t h[4 * kTcUnits], l[4 * kTcUnits];
#pragma unroll
            for (int u = 0; u < kTcUnits; ++u) {
                const int ku = k0 + 8 * u;
                if (WSMEM) {
                    if (have_row && ku < L.cols) wr[u].template load<true>(wrow, L, ku);
                } else {
                    if (have_row && ku + kTcK < L.cols) wn[u].load(wrow, L, ku + kTcK);
                }
                float v[8];
                if (have_row && ku < L.cols) {
                    wr[u].decode(ku, v);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = 0.f;
                }
                split_words<Raw8<FMT>::kExactLo>(v, h + 4 * u, l + 4 * u);
            }
            if (pending >= 0) {
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(wbar0 + 8u * pending);
            }
            // the MMAs that last read stage buffer s (stage kc - S) are done
            if (round > 0 && !mbar_wait_idle(ebar0 + 8u * s, (uint32_t)((round - 1) & 1))) ok = false;
            if (!__all_sync(kFull, ok)) {
                ok = false;
                pending = -1;
                break;
            }
            tc_fence_after();
            static_assert(kTcUnits % 2 == 0, "stores go 8 columns (two units) at a time");
#pragma unroll
            for (int g = 0; g < kTcUnits / 2; ++g) {
                tmem_st8(lane_addr + (uint32_t)kTcK * s + 8u * g, h + 8 * g);
                tmem_st8(lane_addr + (uint32_t)kTcK * s + kTcK / 2 + 8u * g, l + 8 * g);
            }
            pending = s;
            if (!WSMEM) {
#pragma unroll
                for (int u = 0; u < kTcUnits; ++u) wr[u] = wn[u];
            }
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        if (pending >= 0) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(wbar0 + 8u * pending);
        }
    }

    // every MMA has completed once the last stage's commit has arrived
    if (ok && (warp < kDecodeWarps || lane == 0)) {
        const int last = nloc - 1;
        if (!mbar_wait_idle(ebar0 + 8u * (last % S), (uint32_t)((last / S) & 1))) ok = false;
    }
    const bool failed = __syncthreads_or(!ok);
    if (failed && warp == kCopyWarp && lane == 0) {
        report_status(call_status, kStatusMmaTimeout);
        // copies still in flight must land before the CTA exits
        if (WSMEM && !mbar_wait(tbar, 0u)) report_status(call_status, kStatusDrainTimeout);
        for (int j = issued - S > 0 ? issued - S : 0; j < issued; ++j) {
            if (!mbar_wait(xbar0 + 8u * (j % S), (uint32_t)((j / S) & 1))) {
                report_status(call_status, kStatusDrainTimeout);
                break;
            }
        }
    }
    tc_fence_after();
    bool nonfinite = false;
    if (!failed && warp < kDecodeWarps) {
        // warp w reads lanes 32 (w % 4) .. + 31; the four warps sharing a lane
        // quarter take 8-column chunks round-robin
        const int q = warp & 3;
        const int row = r0 + 32 * q + lane;
        for (int c = 8 * (warp >> 2); c < TN; c += 8 * (kDecodeWarps / 4)) {
            float v[8];
            tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < L.rows) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int pos = p0 + c + i;
                    if (pos < np) {
                        Y[(size_t)pos * L.rows + row] = v[i];
                        nonfinite |= !isfinite(v[i]);
                    }
                }
            }
        }
    }
    // A non-finite weight or x makes the split planes NaN: recompute the
    // tile in fp32 (this overwrites every output the epilogue wrote).
    if (__syncthreads_or(nonfinite) && !failed)
        tc_tile_fallback<FMT>(L, w, X, np, Y, r0, p0, TN, kc0 * kTcK, min(kc1 * kTcK, L.cols));
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u));
    }
}

// ------------------------------------------------------------- argmax

__global__ void __launch_bounds__(kThreads)
argmax_kernel(const float *__restrict__ logits, int n, ArgmaxOut am)
{
    __shared__ unsigned long long kscratch[kThreads / 32];
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        best = max_ull(best, make_key(__ldg(logits + i), am.index_base + i));
    best = block_max_key(best, kscratch);
    finish_argmax(best, am, kscratch);
}

// ----------------------------------------------------- repack / dequant

__device__ __forceinline__ void copy16(uint8_t *dst, const uint8_t *src)
{
    for (int k = 0; k < 16; ++k) dst[k] = src[k];
}

// One thread per (row, chunk): move the chunk's bytes from its raw GGUF
// block(s) to their chunk-major places.
__global__ void repack_kernel(Layout L, const uint8_t *__restrict__ raw, uint8_t *__restrict__ dst)
{
    const uint64_t total = (uint64_t)L.rows * L.C;
    const int bb = (L.type == kQ8_0) ? 34 : (L.type == kQ5_0) ? 22 : (L.type == kQ4_K) ? 144 : 210;
    const int C = L.C;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = e / C;
        const int c = (int)(e % C);
        const uint8_t *src = raw + row * (uint64_t)L.nb * bb;
        uint8_t *r = dst + row * L.row_stride;
        switch (L.type) {
        case kQ8_0: {
            const uint8_t *blk = src + (uint64_t)c * 34;
            copy16(r + (c << 4), blk + 2);
            copy16(r + ((C + c) << 4), blk + 18);
            r[L.off_a + 2 * c] = blk[0];
            r[L.off_a + 2 * c + 1] = blk[1];
            break;
        }
        case kQ5_0: {
            const uint8_t *blk = src + (uint64_t)c * 22;
            copy16(r + (c << 4), blk + 6);
            for (int k = 0; k < 4; ++k) r[L.off_a + 4 * c + k] = blk[2 + k];
            r[L.off_b + 2 * c] = blk[0];
            r[L.off_b + 2 * c + 1] = blk[1];
            break;
        }
        case kQ4_K: {
            const int sb = c >> 2, g = c & 3;
            const uint8_t *blk = src + (uint64_t)sb * 144;
            copy16(r + (c << 4), blk + 16 + 32 * g);
            copy16(r + ((C + c) << 4), blk + 32 + 32 * g);
            if (g == 0) copy16(r + L.off_a + (sb << 4), blk);
            break;
        }
        default: {
            const int sb = c >> 2, g = (c >> 1) & 1, h = c & 1;
            const uint8_t *blk = src + (uint64_t)sb * 210;
            copy16(r + (c << 4), blk + 64 * g + 16 * h);
            copy16(r + ((C + c) << 4), blk + 64 * g + 32 + 16 * h);
            copy16(r + ((2 * C + c) << 4), blk + 128 + 32 * g + 16 * h);
            for (int q = 0; q < 4; ++q) r[L.off_a + 4 * c + q] = blk[192 + 8 * g + 2 * q + h];
            if ((c & 3) == 0) {
                r[L.off_b + 2 * sb] = blk[208];
                r[L.off_b + 2 * sb + 1] = blk[209];
            }
            break;
        }
        }
    }
}

// Rebuild the raw GGUF bytes of block b of a resident row (inverse of repack).
__device__ void gather_raw_block(const Layout &L, const uint8_t *r, int b, uint8_t *out)
{
    const int C = L.C;
    switch (L.type) {
    case kQ8_0:
        out[0] = r[L.off_a + 2 * b];
        out[1] = r[L.off_a + 2 * b + 1];
        copy16(out + 2, r + (b << 4));
        copy16(out + 18, r + ((C + b) << 4));
        break;
    case kQ5_0:
        out[0] = r[L.off_b + 2 * b];
        out[1] = r[L.off_b + 2 * b + 1];
        for (int k = 0; k < 4; ++k) out[2 + k] = r[L.off_a + 4 * b + k];
        copy16(out + 6, r + (b << 4));
        break;
    case kQ4_K:
        copy16(out, r + L.off_a + (b << 4));
        for (int g = 0; g < 4; ++g) {
            copy16(out + 16 + 32 * g, r + ((4 * b + g) << 4));
            copy16(out + 32 + 32 * g, r + ((C + 4 * b + g) << 4));
        }
        break;
    default:
        for (int g = 0; g < 2; ++g) {
            for (int h = 0; h < 2; ++h) {
                const int c = 4 * b + 2 * g + h;
                copy16(out + 64 * g + 16 * h, r + (c << 4));
                copy16(out + 64 * g + 32 + 16 * h, r + ((C + c) << 4));
                copy16(out + 128 + 32 * g + 16 * h, r + ((2 * C + c) << 4));
                for (int q = 0; q < 4; ++q) out[192 + 8 * g + 2 * q + h] = r[L.off_a + 4 * c + q];
            }
        }
        out[208] = r[L.off_b + 2 * b];
        out[209] = r[L.off_b + 2 * b + 1];
        break;
    }
}

// The reference's scalar build runs on x86 SSE, where a NaN result carries
// the payload of the first NaN operand (quieted) and an invalid operation on
// non-NaN operands (Inf * 0, Inf - Inf) yields the default NaN 0xFFC00000.
// GPU arithmetic returns a canonical NaN instead, so the dequantiser restores
// the x86 bits to stay bit-exact for every encoding.
__device__ __forceinline__ float x86_nan(float a, float b)
{
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xffc00000u);
}

__device__ __forceinline__ float mul_ref(float a, float b)
{
    const float r = __fmul_rn(a, b);
    return isnan(r) ? x86_nan(a, b) : r;
}

__device__ __forceinline__ float sub_ref(float a, float b)
{
    const float r = __fsub_rn(a, b);
    return isnan(r) ? x86_nan(a, b) : r;
}

__device__ __forceinline__ uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// Value i of a raw GGUF block, with the reference's rounding sequence.
template <uint32_t FMT>
__device__ __forceinline__ float dequant_value(const uint8_t *blk, int i)
{
    if constexpr (FMT == kQ8_0) {
        return mul_ref(f16_exact(rd16(blk)), (float)(int8_t)blk[2 + i]);
    } else if constexpr (FMT == kQ5_0) {
        const uint8_t *qh = blk + 2, *qs = blk + 6;
        const int nib = i < 16 ? (qs[i] & 0x0f) : (qs[i - 16] >> 4);
        const int hi = (qh[i >> 3] >> (i & 7)) & 1;
        return mul_ref(f16_exact(rd16(blk)), (float)((nib | (hi << 4)) - 16));
    } else if constexpr (FMT == kQ4_K) {
        const uint8_t *sm = blk + 4;
        const int j = i >> 5, o = i & 31;
        int sc, mn;
        if (j < 4) {
            sc = sm[j] & 63;
            mn = sm[j + 4] & 63;
        } else {
            sc = (sm[j + 4] & 0x0f) | ((sm[j - 4] >> 6) << 4);
            mn = (sm[j + 4] >> 4) | ((sm[j] >> 6) << 4);
        }
        const float scale = mul_ref(f16_exact(rd16(blk)), (float)sc);
        const float minimum = mul_ref(f16_exact(rd16(blk + 2)), (float)mn);
        const int nib = (blk[16 + 32 * (j >> 1) + o] >> (4 * (j & 1))) & 0x0f;
        return sub_ref(mul_ref(scale, (float)nib), minimum);
    } else {
        const int g = i >> 7, loc = i & 127, r = loc >> 5, o = loc & 31;
        const int lo = (blk[64 * g + 32 * (r & 1) + o] >> (4 * (r >> 1))) & 0x0f;
        const int hi = (blk[128 + 32 * g + o] >> (2 * r)) & 0x03;
        const int q = (lo | (hi << 4)) - 32;
        const int sc = (int8_t)blk[192 + 8 * g + 2 * r + (o >> 4)];
        return mul_ref(mul_ref(f16_exact(rd16(blk + 208)), (float)sc), (float)q);
    }
}

template <uint32_t FMT> struct BlockShape;
template <> struct BlockShape<kQ8_0> { static constexpr int E = 32, B = 34; };
template <> struct BlockShape<kQ5_0> { static constexpr int E = 32, B = 22; };
template <> struct BlockShape<kQ4_K> { static constexpr int E = 256, B = 144; };
template <> struct BlockShape<kQ6_K> { static constexpr int E = 256, B = 210; };

// One thread per block: gather its raw bytes, then decode every value.
template <uint32_t FMT>
__global__ void dequant_layout_kernel(Layout L, const uint8_t *__restrict__ w, float *__restrict__ out)
{
    constexpr int BE = BlockShape<FMT>::E;
    const uint64_t total = (uint64_t)L.rows * L.nb;
    uint8_t raw[BlockShape<FMT>::B];
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = e / L.nb;
        const int b = (int)(e % L.nb);
        gather_raw_block(L, w + row * L.row_stride, b, raw);
        float *o = out + e * BE;
        for (int i = 0; i < BE; ++i) o[i] = dequant_value<FMT>(raw, i);
    }
}

template <uint32_t FMT>
__global__ void dequant_raw_kernel(const uint8_t *__restrict__ raw, uint64_t nblocks, float *__restrict__ out)
{
    constexpr int BE = BlockShape<FMT>::E, BB = BlockShape<FMT>::B;
    const uint64_t total = nblocks * BE;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x)
        out[e] = dequant_value<FMT>(raw + (e / BE) * BB, (int)(e % BE));
}

// ------------------------------------------------- Qwen2 decode step
//
// Kernels of the device-resident decode step (the reference's
// qwen2_forward_token_cached_impl, src/qwen2_architecture.cpp:1195-1531); the
// projections are the fused GEMVs above.  Position and token live in device
// memory (DecodeState), so one step replays from a CUDA graph: embed_kernel
// reads the token, attention_kernel the position, and advance_kernel turns
// the step's argmax key into the next token and moves the position on.  Every
// device-side index is checked: a bad token or a full context sets a bit of
// DecodeState::error and nothing is written out of bounds.

constexpr int kAttnChunk = 64;  // cached tokens per attention CTA
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxGroup = 16;  // query heads per KV head
// merge weights (chunk, head) that fit the score tile: one merge tile
constexpr int kAttnMaxChunks = kAttnMaxGroup * kAttnChunk;

// One CTA: row st->tok of the resident embedding (src/qwen2_architecture.cpp:375-475
// decodes the row with the block dequantiser; same bits here).
template <uint32_t FMT>
__global__ void embed_kernel(Layout L, const uint8_t *__restrict__ w, DecodeState *st, float *__restrict__ h)
{
    constexpr int BE = BlockShape<FMT>::E;
    int tok = st->tok;
    if (tok < 0 || tok >= L.rows) {
        if (threadIdx.x == 0) atomicOr(&st->error, 1u);
        tok = 0;
    }
    uint8_t raw[BlockShape<FMT>::B];
    for (int b = threadIdx.x; b < L.nb; b += blockDim.x) {
        gather_raw_block(L, w + (uint64_t)tok * L.row_stride, b, raw);
        for (int i = 0; i < BE; ++i) h[b * BE + i] = dequant_value<FMT>(raw, i);
    }
}

// Grid (kv head g, chunk c of kAttnChunk cached tokens).  Each CTA rotates the
// query heads of group g (transformer_apply_rope_f32, src/transformer_ops.cpp:16-66:
// pairs (i, i + hd/2), angle = pos / base^(2i/hd)), and, when its chunk holds
// the new position, rotates that key and appends key and value to the cache.
// It then forms its chunk's scores q.k / sqrt(hd), their maximum m, the sum l
// of exp(score - m) and the weighted value sum o, and stores (m, l, o).  The
// last CTA of group g to arrive merges the chunks: out = sum_c e^(m_c - M) o_c /
// sum_c e^(m_c - M) l_c -- the softmax and weighted sum of
// transformer_attention_f32 (src/transformer_ops.cpp:68-153), evaluated
// chunk-wise.
// Shared tiles of one attention work item.
template <int HD>
struct AttnShared {
    float cs[HD / 2], sn[HD / 2];
    float qs[kAttnMaxGroup][HD];
    float ks[kAttnChunk][HD + 1];
    __align__(16) float vs[kAttnChunk][HD];
    float sc[kAttnMaxGroup][kAttnChunk];
    float mx[kAttnMaxGroup], den[kAttnMaxGroup];
    int last;
};

// One work item (kv head g, chunk c) of the decode attention, run by all NT
// threads of the CTA.  PDL: the
// standalone kernel's programmatic-launch handshake around the loads that do
// not depend on the Q/K/V projection.
template <int HD, bool PDL, int NT = kAttnThreads>
__device__ void attention_item(AttnShared<HD> &sm, int g, int c, const float *__restrict__ qkv, int heads,
                               int kv_heads, float *__restrict__ kc, float *__restrict__ vc, int max_ctx,
                               float rope_base, const DecodeState *st, float *__restrict__ part,
                               unsigned int *__restrict__ counter, float *__restrict__ att)
{
    auto &cs = sm.cs;
    auto &sn = sm.sn;
    auto &qs = sm.qs;
    auto &ks = sm.ks;
    auto &vs = sm.vs;
    auto &sc = sm.sc;
    auto &last = sm.last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = st->pos;
    const int T = pos + 1, nchunk = (T + kAttnChunk - 1) / kAttnChunk;
    const int G = heads / kv_heads, dim = heads * HD, kvd = kv_heads * HD;
    const int t0 = c * kAttnChunk, tn = min(kAttnChunk, T - t0);

    // Cached positions (< pos) do not depend on this layer's projections:
    // load them before waiting for the Q/K/V GEMV, every load in flight at once.
    constexpr int kV4 = kAttnChunk * HD / 4 / NT;  // float4 per thread per matrix
    static_assert(kAttnChunk * HD % (4 * NT) == 0, "whole float4 per thread");
    float4 kr4[kV4], vr4[kV4];
#pragma unroll
    for (int i = 0; i < kV4; ++i) {
        const int e4 = tid + i * NT, t = (4 * e4) / HD, d = (4 * e4) % HD, tok = t0 + t;
        const size_t slot = (size_t)tok * kvd + g * HD + d;
        if (t < tn && tok != pos) {
            kr4[i] = __ldg(reinterpret_cast<const float4 *>(kc + slot));
            vr4[i] = __ldg(reinterpret_cast<const float4 *>(vc + slot));
        }
    }
    if (tid < HD / 2) {
        const float angle = (float)pos / powf(rope_base, (2.0f * (float)tid / (float)HD));
        cs[tid] = cosf(angle);
        sn[tid] = sinf(angle);
    }
#pragma unroll
    for (int i = 0; i < kV4; ++i) {
        const int e4 = tid + i * NT, t = (4 * e4) / HD, d = (4 * e4) % HD, tok = t0 + t;
        if (t < tn && tok != pos) {
            ks[t][d] = kr4[i].x; ks[t][d + 1] = kr4[i].y; ks[t][d + 2] = kr4[i].z; ks[t][d + 3] = kr4[i].w;
            *reinterpret_cast<float4 *>(&vs[t][d]) = vr4[i];
        }
    }
    // q, k and v of this position come from the Q/K/V GEMV
    if constexpr (PDL) asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    for (int e = tid; e < G * HD; e += NT) {
        const int hh = e / HD, d = e % HD, i = d % (HD / 2);
        const float *q = qkv + (g * G + hh) * HD;
        const float x = __ldcg(q + i), y = __ldcg(q + i + HD / 2);
        qs[hh][d] = d < HD / 2 ? x * cs[i] - y * sn[i] : x * sn[i] + y * cs[i];
    }
    if (pos >= t0 && pos < t0 + tn) {
        const int t = pos - t0;
        for (int d = tid; d < HD; d += NT) {
            const int i = d % (HD / 2);
            const float *k = qkv + dim + g * HD;
            const float x = __ldcg(k + i), y = __ldcg(k + i + HD / 2);
            const float kr = d < HD / 2 ? x * cs[i] - y * sn[i] : x * sn[i] + y * cs[i];
            const float vv = __ldcg(qkv + dim + kvd + g * HD + d);
            const size_t slot = (size_t)pos * kvd + g * HD + d;
            kc[slot] = kr;
            vc[slot] = vv;
            ks[t][d] = kr;
            vs[t][d] = vv;
        }
    }
    __syncthreads();
    const float rs = sqrtf((float)HD);
    for (int e = tid; e < G * tn; e += NT) {
        const int hh = e / tn, t = e % tn;
        float acc = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; ++d) acc += qs[hh][d] * ks[t][d];
        sc[hh][t] = acc / rs;
    }
    __syncthreads();
    float *pc = part + ((size_t)(g * ((max_ctx + kAttnChunk - 1) / kAttnChunk) + c) * G) * (HD + 2);
    for (int hh = warp; hh < G; hh += NT / 32) {
        float m = -INFINITY;
        for (int t = lane; t < tn; t += 32) m = fmaxf(m, sc[hh][t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
        float l = 0.f;
        for (int t = lane; t < tn; t += 32) {
            const float p = expf(sc[hh][t] - m);
            sc[hh][t] = p;
            l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(kFull, l, o);
        if (lane == 0) {
            pc[hh * (HD + 2)] = m;
            pc[hh * (HD + 2) + 1] = l;
        }
    }
    __syncthreads();
    for (int e = tid; e < G * HD; e += NT) {
        const int hh = e / HD, d = e % HD;
        float o = 0.f;
        for (int t = 0; t < tn; ++t) o += sc[hh][t] * vs[t][d];
        pc[hh * (HD + 2) + 2 + d] = o;
    }
    // the last CTA of this group to finish merges every chunk
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&counter[g], 1u) == (unsigned)(nchunk - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // Merge: the weights e^(m_c - M) once per (chunk, head), the denominators
    // sum_c e^(m_c - M) l_c, then the weighted output sums with independent
    // loads.
    const float *pg = part + (size_t)g * ((max_ctx + kAttnChunk - 1) / kAttnChunk) * G * (HD + 2);
    // The chunks are merged in tiles whose G weights each fit the score tile,
    // so any context length merges (one tile up to kAttnMaxChunks / G chunks).
    float *wgt = &sc[0][0];
    auto &mx = sm.mx;
    auto &den = sm.den;
    const int tile = kAttnMaxChunks / G;
    // pass 1: the maximum of every head's chunk maxima
    if (tid < G) mx[tid] = -INFINITY;
    for (int k0 = 0; k0 < nchunk; k0 += tile) {
        const int nk = min(tile, nchunk - k0);
        __syncthreads();
        for (int e = tid; e < nk * G; e += NT) wgt[e] = __ldcg(pg + ((size_t)k0 * G + e) * (HD + 2));
        __syncthreads();
        if (tid < G) {
            float M = mx[tid];
            for (int k = 0; k < nk; ++k) M = fmaxf(M, wgt[k * G + tid]);
            mx[tid] = M;
        }
    }
    // pass 2: weights e^(m_c - M), the denominators and the weighted sums
    constexpr int kOut = (kAttnMaxGroup * HD + NT - 1) / NT;  // outputs per thread
    float o[kOut];
#pragma unroll
    for (int j = 0; j < kOut; ++j) o[j] = 0.f;
    if (tid < G) den[tid] = 0.f;
    for (int k0 = 0; k0 < nchunk; k0 += tile) {
        const int nk = min(tile, nchunk - k0);
        __syncthreads();
        for (int e = tid; e < nk * G; e += NT)
            wgt[e] = expf(__ldcg(pg + ((size_t)k0 * G + e) * (HD + 2)) - mx[e % G]);
        __syncthreads();
        for (int hh = warp; hh < G; hh += NT / 32) {
            float l = 0.f;
            for (int k = lane; k < nk; k += 32)
                l += wgt[k * G + hh] * __ldcg(pg + ((size_t)(k0 + k) * G + hh) * (HD + 2) + 1);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(kFull, l, off);
            if (lane == 0) den[hh] += l;
        }
#pragma unroll
        for (int j = 0; j < kOut; ++j) {
            const int e = tid + j * NT;
            if (e < G * HD) {
                const int hh = e / HD, d = e % HD;
#pragma unroll 8
                for (int k = 0; k < nk; ++k)
                    o[j] += wgt[k * G + hh] * __ldcg(pg + ((size_t)(k0 + k) * G + hh) * (HD + 2) + 2 + d);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kOut; ++j) {
        const int e = tid + j * NT;
        if (e < G * HD) att[(g * G + e / HD) * HD + e % HD] = o[j] / den[e / HD];
    }
    if (tid == 0) counter[g] = 0u;
}

// Grid (kv head g, chunk c of kAttnChunk cached tokens): one work item per CTA.
template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
attention_kernel(const float *__restrict__ qkv, int heads, int kv_heads, float *__restrict__ kc,
                 float *__restrict__ vc, int max_ctx, float rope_base, DecodeState *st, float *__restrict__ part,
                 unsigned int *__restrict__ counter, float *__restrict__ att)
{
    __shared__ AttnShared<HD> sm;
    const int g = blockIdx.x, c = blockIdx.y;
    // The next launch (the output projection) may start streaming its
    // weights; it reads att only after its own griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int pos = st->pos;  // written by the previous step's advance_kernel
    if (pos < 0 || pos >= max_ctx) {
        if (g == 0 && c == 0 && threadIdx.x == 0) atomicOr(&st->error, 2u);
        return;
    }
    if (c >= (pos + kAttnChunk) / kAttnChunk) return;  // chunk beyond the position
    attention_item<HD, true>(sm, g, c, qkv, heads, kv_heads, kc, vc, max_ctx, rope_base, st, part, counter, att);
}

// ------------------------------------- decode attention on a CTA cluster
//
// One cluster of kDaSplit CTAs per KV head and part of its query-head group
// (groups of 4 or more query heads are split in two parts, so each CTA scores
// half the heads).  CTA r of the cluster owns the positions [r*T/S,
// (r+1)*T/S) of the T = pos + 1 positions and the part's query heads (a
// group of G <= 8): it stages its cached keys and values in shared
// memory with 16-byte cp.async copies before griddepcontrol.wait (they do not
// depend on this layer's projections, so the copies overlap the Q/K/V GEMV),
// then rotates the group's queries, computes its scores, softmax and weighted
// value sums over tiles of kDaTile positions (online softmax across tiles:
// running maximum m, sum of exponentials l, weighted sum o), and sends
// {m, l, o[64]} per head to the leader CTA with asynchronous remote stores
// (st.async into the leader's shared memory, completing on the leader's
// mbarrier).  The leader merges the S partials per head as
// sum_r e^(m_r - M) o_r / sum_r e^(m_r - M) l_r -- the softmax and weighted
// sum of transformer_attention_f32 (src/transformer_ops.cpp:68-153)
// evaluated over position ranges.  The CTA whose range ends at pos rotates
// this position's key, appends key and value to the cache, and patches them
// into its staged tile.  The only cluster barrier (it orders the leader's
// mbarrier initialisation before the remote stores) is arrived at before
// griddepcontrol.wait, so it is off the critical path; the leader's wait is
// bounded (2 s, then decode-state error bit 16).
constexpr int kDaSplit = 16;
constexpr int kDaTile = 128;       // positions per staged tile
constexpr int kDaThreads = 256;    // 8 warps: warp h runs head h's softmax and weighted sums
constexpr int kDaMaxGroup = 8;
constexpr int kDaKStride = 68;     // floats per staged key row: conflict-free 128-bit reads
constexpr int kDaPart = 68;        // floats per received partial: m, l, 2 pad, o[64] (16-byte aligned o)
constexpr uint32_t kDaKBytes = kDaTile * kDaKStride * 4;
constexpr uint32_t kDaVBytes = kDaTile * 64 * 4;
constexpr uint32_t kDaPartBytes = kDaSplit * kDaMaxGroup * kDaPart * 4;
constexpr uint32_t kDaSmem =
    kDaKBytes + kDaVBytes + kDaMaxGroup * 64 * 4 + kDaMaxGroup * kDaTile * 4 + 2 * 64 * 4 + kDaPartBytes;

__device__ __forceinline__ void da_cp16(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Stage keys/values of positions [a, b) (b - a <= kDaTile) of KV head g,
// skipping position `skip` (not yet written).
__device__ __forceinline__ void da_stage(float *ks, float *vs, const float *kc, const float *vc, int kvd, int g, int a,
                                         int b, int skip)
{
    const uint32_t ks_a = (uint32_t)__cvta_generic_to_shared(ks), vs_a = (uint32_t)__cvta_generic_to_shared(vs);
    const int n16 = (b - a) * 16;  // 16-byte pieces per matrix
    for (int e = threadIdx.x; e < 2 * n16; e += kDaThreads) {
        const int m = e >= n16, f = e - m * n16, t = f >> 4, q = f & 15;
        if (a + t == skip) continue;
        const size_t src = (size_t)(a + t) * kvd + g * 64 + q * 4;
        if (m == 0)
            da_cp16(ks_a + (uint32_t)(t * kDaKStride + q * 4) * 4u, kc + src);
        else
            da_cp16(vs_a + (uint32_t)(t * 64 + q * 4) * 4u, vc + src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(kDaThreads, 1)
attention_cluster_kernel(const float *__restrict__ qkv, int heads, int kv_heads, float *__restrict__ kc,
                         float *__restrict__ vc, int max_ctx, float rope_base, DecodeState *st,
                         float *__restrict__ att, int hsplit)
{
    extern __shared__ __align__(128) uint8_t smem[];
    float *ks = reinterpret_cast<float *>(smem);                          // [kDaTile][kDaKStride]
    float *vs = reinterpret_cast<float *>(smem + kDaKBytes);              // [kDaTile][64]
    float *qs = reinterpret_cast<float *>(smem + kDaKBytes + kDaVBytes);  // [Gs][64]
    float *ps = qs + kDaMaxGroup * 64;                                    // [Gs][kDaTile]
    float *knew = ps + kDaMaxGroup * kDaTile;                             // rotated key of pos [64], value [64]
    float *part = knew + 128;                                             // leader: [S][kDaMaxGroup][kDaPart]
    __shared__ float cs[32], sn[32], mh[kDaMaxGroup], lh[kDaMaxGroup];
    __shared__ float wr[kDaSplit][kDaMaxGroup];
    __shared__ __align__(8) unsigned long long bar;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    // cluster (KV head g, head part hs): query heads [h0, h0 + Gs) of the group
    const int cid = (int)(blockIdx.x / kDaSplit), g = cid / hsplit, hs = cid % hsplit;
    const int G = heads / kv_heads, dim = heads * 64, kvd = kv_heads * 64;
    const int h0 = hs * G / hsplit, Gs = (hs + 1) * G / hsplit - h0;
    const uint32_t bar_a = (uint32_t)__cvta_generic_to_shared(&bar);
    // The output projection may start copying its weights; it reads att only
    // after its own griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int pos = st->pos;  // written by the previous step's advance kernel
    if (pos < 0 || pos >= max_ctx) {  // the same for every CTA: no cluster barrier is reached
        if (blockIdx.x == 0 && tid == 0) atomicOr(&st->error, 2u);
        return;
    }
    if (rank == 0 && tid == 0) {
        // the leader's mbarrier expects the other CTAs' partials
        mbar_init(bar_a, 1u);
        mbar_expect_tx(bar_a, (uint32_t)((kDaSplit - 1) * Gs * (64 + 2) * 4));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int T = pos + 1;
    const int a0 = (int)((long long)T * rank / kDaSplit), b0 = (int)((long long)T * (rank + 1) / kDaSplit);
    const int ntiles = (b0 - a0 + kDaTile - 1) / kDaTile;
    if (ntiles > 0) da_stage(ks, vs, kc, vc, kvd, g, a0, min(b0, a0 + kDaTile), pos);
    if (tid < 32) {
        const float angle = (float)pos / powf(rope_base, (2.0f * (float)tid / 64.f));
        cs[tid] = cosf(angle);
        sn[tid] = sinf(angle);
    }
    if (tid < kDaMaxGroup) {
        mh[tid] = -INFINITY;
        lh[tid] = 0.f;
    }
    // q, k and v of this position come from the Q/K/V GEMV
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    for (int e = tid; e < Gs * 64; e += kDaThreads) {
        const int hh = e >> 6, d = e & 63, i = d & 31;
        const float *q = qkv + (g * G + h0 + hh) * 64;
        const float x = __ldcg(q + i), y = __ldcg(q + i + 32);
        qs[hh * 64 + d] = d < 32 ? x * cs[i] - y * sn[i] : x * sn[i] + y * cs[i];
    }
    const bool owns_pos = pos >= a0 && pos < b0;
    if (owns_pos && tid < 64) {
        const int d = tid, i = d & 31;
        const float *k = qkv + dim + g * 64;
        const float x = __ldcg(k + i), y = __ldcg(k + i + 32);
        const float kr = d < 32 ? x * cs[i] - y * sn[i] : x * sn[i] + y * cs[i];
        const float vv = __ldcg(qkv + dim + kvd + g * 64 + d);
        const size_t slot = (size_t)pos * kvd + g * 64 + d;
        if (hs == 0) {  // one cluster of the KV head appends to the cache
            kc[slot] = kr;
            vc[slot] = vv;
        }
        knew[d] = kr;
        knew[64 + d] = vv;
    }
    // per thread: the weighted sums of head `warp`, dimensions 4*(lane & 15)..,
    // over the tile positions of half (lane >> 4)
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    const int dq = lane & 15, half = lane >> 4;
    const float rs = sqrtf(64.f);
    for (int ti = 0; ti < ntiles; ++ti) {
        const int a = a0 + ti * kDaTile, b = min(b0, a + kDaTile), tn = b - a;
        if (ti > 0) {
            __syncthreads();  // every thread is done with the previous tile
            da_stage(ks, vs, kc, vc, kvd, g, a, b, pos);
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        if (pos >= a && pos < b && tid < 64) {  // this position's key and value
            ks[(pos - a) * kDaKStride + tid] = knew[tid];
            vs[(pos - a) * 64 + tid] = knew[64 + tid];
        }
        __syncthreads();
        // scores: thread (position t, heads hg, hg + NG, ...): NG = 4 groups
        // of 64 positions when the tile has at most 64, else 2 of 128
        {
            const int P = tn <= 64 ? 64 : kDaTile, NG = kDaThreads / P;
            const int t = tid % P, hg = tid / P;
            if (t < tn) {
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                const float4 *kr = reinterpret_cast<const float4 *>(ks + t * kDaKStride);
#pragma unroll 4
                for (int d4 = 0; d4 < 16; ++d4) {
                    const float4 k4 = kr[d4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int hh = hg + NG * j;
                        if (hh < Gs) {
                            const float4 q4 = reinterpret_cast<const float4 *>(qs + hh * 64)[d4];
                            acc[j] += q4.x * k4.x;
                            acc[j] += q4.y * k4.y;
                            acc[j] += q4.z * k4.z;
                            acc[j] += q4.w * k4.w;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (hg + NG * j < Gs) ps[(hg + NG * j) * kDaTile + t] = acc[j] / rs;
            }
        }
        __syncthreads();
        // softmax update of head `warp`: running maximum and sum, tile weights
        if (warp < Gs) {
            float *pr = ps + warp * kDaTile;
            float mt = -INFINITY;
            for (int t = lane; t < tn; t += 32) mt = fmaxf(mt, pr[t]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(kFull, mt, off));
            const float m_old = mh[warp], m_new = fmaxf(m_old, mt);
            float l = 0.f;
            for (int t = lane; t < tn; t += 32) {
                const float p = expf(pr[t] - m_new);
                pr[t] = p;
                l += p;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(kFull, l, off);
            const float alpha = expf(m_old - m_new);  // 0 on the first tile
            __syncwarp();
            if (lane == 0) {
                mh[warp] = m_new;
                lh[warp] = lh[warp] * alpha + l;
            }
            // weighted value sums of this head (the warp owns it)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] *= alpha;
            const int t_end = min(tn, (half + 1) * (kDaTile / 2));
#pragma unroll 8
            for (int t = half * (kDaTile / 2); t < t_end; ++t) {
                const float p = pr[t];
                const float4 v4 = reinterpret_cast<const float4 *>(vs + t * 64)[dq];
                o[0] += p * v4.x;
                o[1] += p * v4.y;
                o[2] += p * v4.z;
                o[3] += p * v4.w;
            }
            __syncwarp();
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] += __shfl_xor_sync(kFull, o[j], 16);
    __syncthreads();  // mh / lh final
    // the leader's mbarrier is initialised (cluster barrier arrived at above)
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    if (warp < Gs) {
        float *mine = part + (rank * kDaMaxGroup + warp) * kDaPart;
        if (rank == 0) {
            if (lane < 16) *reinterpret_cast<float4 *>(mine + 4 + 4 * dq) = make_float4(o[0], o[1], o[2], o[3]);
            if (lane == 0) *reinterpret_cast<float2 *>(mine) = make_float2(mh[warp], lh[warp]);
        } else {
            uint32_t remote, rbar;
            const uint32_t local = (uint32_t)__cvta_generic_to_shared(mine);
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(local));
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(rbar) : "r"(bar_a));
            if (lane < 16)
                asm volatile(
                    "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                        remote + 16u + 16u * (uint32_t)dq),
                    "f"(o[0]), "f"(o[1]), "f"(o[2]), "f"(o[3]), "r"(rbar)
                    : "memory");
            if (lane == 0)
                asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                                 remote),
                             "f"(mh[warp]), "f"(lh[warp]), "r"(rbar)
                             : "memory");
        }
    }
    if (rank != 0) return;
    // leader: every partial has landed (bounded wait; the barrier also
    // publishes the leader's own partials), then the merge
    const bool landed = mbar_wait(bar_a, 0u);
    if (!__syncthreads_and(landed)) {
        if (tid == 0) atomicOr(&st->error, 16u);
        return;
    }
    if (tid < Gs) {
        float M = -INFINITY;
        for (int r = 0; r < kDaSplit; ++r) M = fmaxf(M, part[(r * kDaMaxGroup + tid) * kDaPart]);
        float den = 0.f;
        for (int r = 0; r < kDaSplit; ++r) {
            const float w = expf(part[(r * kDaMaxGroup + tid) * kDaPart] - M);
            wr[r][tid] = w;
            den += w * part[(r * kDaMaxGroup + tid) * kDaPart + 1];
        }
        lh[tid] = den;
    }
    __syncthreads();
    for (int e = tid; e < Gs * 64; e += kDaThreads) {
        const int hh = e >> 6, d = e & 63;
        float num = 0.f;
#pragma unroll 4
        for (int r = 0; r < kDaSplit; ++r) num += wr[r][hh] * part[(r * kDaMaxGroup + hh) * kDaPart + 4 + d];
        att[(g * G + h0 + hh) * 64 + d] = num / lh[hh];
    }
}

// One thread: the step's greedy token (key of index_base 0) becomes the next
// step's input; the position moves on.
__global__ void advance_kernel(const unsigned long long *key, DecodeState *st, int *history, int max_steps,
                               unsigned int *bar_count)
{
    if (bar_count != nullptr) *bar_count = 0u;  // re-arm the persistent step's grid barrier
    const unsigned long long k = *key;
    int tok = 0;
    if (k == 0ull || k == ~0ull)
        atomicOr(&st->error, 4u);
    else
        tok = (int)(0xffffffffu - (unsigned int)(k & 0xffffffffull));
    st->tok = tok;
    if (st->steps >= 0 && st->steps < max_steps) history[st->steps] = tok;
    st->steps += 1;
    st->pos += 1;
}

// ------------------------------------------- persistent decode layers
//
// The whole layer stack of one decode step in one cooperative launch: one CTA
// per SM runs the embedding and, per layer, five phases separated by grid
// barriers --
//   1  [q; k; v] rows of this CTA, RMSNorm(attn_norm) prologue, biases
//   2  attention work items (kv head, 64-token chunk), as attention_kernel
//   3  o rows, residual (h += W_o att)
//   4  [gate; up] rows, RMSNorm(ffn_norm) prologue
//   5  down rows, SwiGLU prologue (up * silu(gate)), residual
// -- instead of five launches whose boundaries each cost a drain, a launch and
// a pipeline fill.  Every CTA owns a fixed row range of every matrix.  The
// projections of the step form one sequence of units (q, k, v or [q; k; v],
// o, gate and up or [gate; up], down, layer after layer); a CTA keeps its rows
// of the next two units in flight into two shared-memory slots (bulk copies
// completing on an mbarrier per slot), so a phase's weights are on chip
// before its barrier opens.  (Bulk L2 prefetches of the layer after were
// tried and dropped: issuing them stalled the issuing thread ~3 us a layer.)
// Rows that do not fit a slot are read from global memory.  The current and
// next layer's descriptors sit in shared memory.  Activations written in the
// launch are read through L2 (ld.global.cg) in one pass: the RMSNorm prologue
// quantizes x * norm and scales the row sums by 1 / sqrt(mean(x^2) + eps),
// and a unit whose x has the slice layout of the previous unit of its phase
// (gate then up, q then k then v) reuses it.  The x quantization and
// block dots are the GEMV kernels'; a row's 32-chunk blocks may sit in
// different warps and are summed in block order.  Barriers count arrivals
// (the advance kernel re-arms the counter after each step) and are bounded:
// one that does not complete within 2 s raises an abort flag that every
// later barrier honours, sets error bit 8 of the decode state and ends the
// launch.

constexpr int kPsThreads = 512;
constexpr int kPsParts = 4096;  // per-CTA partial sums of (row, 32-chunk block) items

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int *p)
{
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned int *p, unsigned int v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier number k of the launch (k = 1, 2, ...): wait until k arrivals
// per CTA have been counted.  false once any CTA's wait has expired.
__device__ bool grid_sync(GridBar *b, unsigned int k, DecodeState *st)
{
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ok = 1;
        const unsigned int target = k * gridDim.x;
        red_release_gpu_add(&b->count, 1u);
        if (ld_acquire_gpu(&b->count) < target) {
            const unsigned long long t0 = globaltimer();
            for (uint32_t n = 1; ld_acquire_gpu(&b->count) < target; ++n) {
                if ((n & 63u) != 0u) continue;
                if (*(volatile unsigned int *)&b->abort) {
                    ok = 0;
                    break;
                }
                if (globaltimer() - t0 > kWaitLimitNs) {
                    atomicExch(&b->abort, 1u);
                    atomicOr(&st->error, 8u);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

__device__ __forceinline__ void cta_rows(int rows, int *r0, int *r1)
{
    *r0 = (int)((long long)rows * blockIdx.x / gridDim.x);
    *r1 = (int)((long long)rows * (blockIdx.x + 1) / gridDim.x);
}

// The step's projections as one sequence of units: per layer q, k, v (or
// [q; k; v]), o, gate, up (or [gate; up]), down.
struct PsUnits {
    const PLayer *ring;  // shared-memory copies of layers l (slot l & 1) and l + 1
    __device__ int per_layer(int l) const { return ring[l & 1].n_qkv + ring[l & 1].n_gu + 2; }
    // unit u of layer l (null past the layer)
    __device__ const PGemv *at(int l, int u) const
    {
        const PLayer &ly = ring[l & 1];
        if (u < ly.n_qkv) return &ly.qkv[u];
        u -= ly.n_qkv;
        if (u == 0) return &ly.o;
        u -= 1;
        if (u < ly.n_gu) return &ly.gu[u];
        u -= ly.n_gu;
        return u == 0 ? &ly.down : nullptr;
    }
};

// Position of the unit that the slots load next (every thread keeps the same
// copy; thread 0 issues).
struct PsCursor {
    int l = 0, u = 0, seq = 0;
};

__device__ __forceinline__ uint64_t unit_bytes(const PGemv &g)
{
    int r0, r1;
    cta_rows(g.L.rows, &r0, &r1);
    return (uint64_t)(r1 - r0) * g.L.row_stride;
}

// Start loading the unit at the cursor into slot seq & 1 and advance the
// cursor.  The slot's mbarrier completes one phase per unit: with the bytes
// of a bulk copy, or at once for a unit that does not fit (read from global).
__device__ void ps_issue(const PStep &P, const PLayer *ring, PsCursor &cur, uint32_t slots, uint32_t slot_bytes,
                         uint32_t bars)
{
    const PsUnits U{ring};
    if (cur.l >= P.n_layers) return;
    const PGemv &g = *U.at(cur.l, cur.u);
    if (threadIdx.x == 0) {
        const uint32_t bar = bars + 8u * (uint32_t)(cur.seq & 1);
        const uint64_t bytes = unit_bytes(g);
        if (bytes > 0 && bytes <= slot_bytes) {
            int r0, r1;
            cta_rows(g.L.rows, &r0, &r1);
            const uint8_t *src = g.w + (uint64_t)r0 * g.L.row_stride;
            const uint32_t dst = slots + (uint32_t)(cur.seq & 1) * slot_bytes;
            mbar_expect_tx(bar, (uint32_t)bytes);
            for (uint32_t off = 0; off < (uint32_t)bytes; off += 32768u)
                bulk_g2s(dst + off, src + off, min(32768u, (uint32_t)bytes - off), bar);
        } else {
            mbar_arrive(bar);
        }
    }
    cur.seq += 1;
    if (++cur.u == U.per_layer(cur.l)) {
        cur.u = 0;
        cur.l += 1;
    }
}

// This CTA's rows of y = W x' (+ add) for the unit of sequence number seq;
// x and add may have been written earlier in the launch.
// reuse: the quantized x in shared memory (and red[], which holds the sum of
// squares) came from the previous unit of this phase, with the same x,
// prologue and slice layout.
template <uint32_t FMT>
__device__ bool ps_gemv(const PGemv &g, int seq, uint32_t slots, uint32_t slot_bytes, uint32_t bars, const float *x,
                        int pre, const float *aux, float eps, float *y, const float *add, uint8_t *smem, float *parts,
                        float *red, GridBar *b, DecodeState *st, bool reuse)
{
    const Layout &L = g.L;
    const int C = L.C, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NSL = W<FMT>::kSlices;
    float scale = 1.f, ss = 0.f;
    if (!reuse) {
        quantize_x<FMT, kPsThreads, true>(x, L.cols, C, smem, 1, 0, pre == kPreRmsNorm ? kPreScale : pre, 1.f, aux,
                                          nullptr, &ss);
        if (pre == kPreRmsNorm) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
            if (lane == 0) red[warp] = ss;
        }
        __syncthreads();
    }
    if (pre == kPreRmsNorm) {
        ss = 0.f;
        for (int i = 0; i < kPsThreads / 32; ++i) ss += red[i];
        scale = 1.f / sqrtf(ss / (float)L.cols + eps);
    }
    const XS s = xs_view(smem, L.cols);
    const uint64_t bytes = unit_bytes(g);
    const bool in_smem = bytes > 0 && bytes <= slot_bytes;
    const uint32_t slot = slots + (uint32_t)(seq & 1) * slot_bytes;
    // every thread waits for the slot (its phase completes even when the
    // unit is read from global memory)
    if (!mbar_wait(bars + 8u * (uint32_t)(seq & 1), (uint32_t)((seq >> 1) & 1))) {
        if (tid == 0) {
            atomicExch(&b->abort, 1u);
            atomicOr(&st->error, 8u);
        }
        return false;
    }
    int r0, r1;
    cta_rows(L.rows, &r0, &r1);
    const int NB = (C + 31) / 32;
    const int RB = max(1, kPsParts / NB);
    for (int rb = r0; rb < r1; rb += RB) {
        const int nr = min(RB, r1 - rb), items = nr * NB;
        for (int it = warp; it < items; it += kPsThreads / 32) {
            const int r = it / NB, bk = it - r * NB, c = bk * 32 + lane;
            float acc = 0.f;
            if (c < C) {
                W<FMT> wv;
                if (in_smem)
                    wv.load_smem(slot + (uint32_t)(rb + r - r0) * (uint32_t)L.row_stride, L, c);
                else
                    wv.load(g.w + (uint64_t)(rb + r) * L.row_stride, L, c);
                const XR<NSL> xr = load_xr<NSL>(s, C, c);
                acc = wv.dot(xr);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
            if (lane == 0) parts[it] = acc;
        }
        __syncthreads();
        for (int r = tid; r < nr; r += kPsThreads) {
            float v = 0.f;
            for (int bk = 0; bk < NB; ++bk) v += parts[r * NB + bk];
            v *= scale;
            const int row = rb + r;
            if (add != nullptr) v += __ldcg(add + row);
            y[row] = v;
        }
        __syncthreads();
    }
    // every thread is past the slot's wait before thread 0 re-arms the slot
    __syncthreads();
    return true;
}

__device__ bool ps_gemv_any(const PGemv &g, int seq, uint32_t slots, uint32_t slot_bytes, uint32_t bars,
                            const float *x, int pre, const float *aux, float eps, float *y, const float *add,
                            uint8_t *smem, float *parts, float *red, GridBar *b, DecodeState *st, bool reuse)
{
    switch (g.L.type) {
    case kQ8_0:
        return ps_gemv<kQ8_0>(g, seq, slots, slot_bytes, bars, x, pre, aux, eps, y, add, smem, parts, red, b, st, reuse);
    case kQ5_0:
        return ps_gemv<kQ5_0>(g, seq, slots, slot_bytes, bars, x, pre, aux, eps, y, add, smem, parts, red, b, st, reuse);
    case kQ4_K:
        return ps_gemv<kQ4_K>(g, seq, slots, slot_bytes, bars, x, pre, aux, eps, y, add, smem, parts, red, b, st, reuse);
    default:
        return ps_gemv<kQ6_K>(g, seq, slots, slot_bytes, bars, x, pre, aux, eps, y, add, smem, parts, red, b, st, reuse);
    }
}

// Formats whose quantized x has the same slice layout (Q8_0 and Q5_0: 16-element
// halves of 32-blocks; Q4_K; Q6_K).
__device__ __forceinline__ int slice_family(uint32_t type) { return type == kQ5_0 ? (int)kQ8_0 : (int)type; }

template <uint32_t FMT>
__device__ void ps_embed(const PGemv &e, int tok, float *h)
{
    constexpr int BE = BlockShape<FMT>::E;
    uint8_t raw[BlockShape<FMT>::B];
    for (int bk = blockIdx.x * blockDim.x + threadIdx.x; bk < e.L.nb; bk += gridDim.x * blockDim.x) {
        gather_raw_block(e.L, e.w + (uint64_t)tok * e.L.row_stride, bk, raw);
        for (int i = 0; i < BE; ++i) h[bk * BE + i] = dequant_value<FMT>(raw, i);
    }
}

// Dynamic shared memory: quantized x | partial sums | two weight slots.
__host__ __device__ constexpr uint32_t ps_x_bytes(int dim, int hid)
{
    return (uint32_t)((xs_bytes(dim > hid ? dim : hid) + 127) / 128 * 128);
}

__global__ void __launch_bounds__(kPsThreads, 1) decode_layers_kernel(PStep P)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ AttnShared<64> attn;
    __shared__ float red[kPsThreads / 32];
    __shared__ __align__(8) unsigned long long slot_bars[2];
    __shared__ __align__(16) PLayer ring[2];  // layers l (slot l & 1) and l + 1
    float *parts = reinterpret_cast<float *>(smem + ps_x_bytes(P.dim, P.hid));
    const uint32_t slots = (uint32_t)__cvta_generic_to_shared(smem + ps_x_bytes(P.dim, P.hid) + 4u * kPsParts);
    const uint32_t bars = (uint32_t)__cvta_generic_to_shared(&slot_bars[0]);
    const int pos = P.st->pos, tok = P.st->tok;
    if (pos < 0 || pos >= P.max_ctx) {  // uniform over the grid: no barrier is reached
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&P.st->error, 2u);
        return;
    }
    // copy layer l's descriptor into ring slot l & 1 (all threads, then a barrier)
    auto load_layer = [&](int l) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(P.layers + l);
        uint32_t *dst = reinterpret_cast<uint32_t *>(&ring[l & 1]);
        for (int i = threadIdx.x; i < (int)(sizeof(PLayer) / 4); i += kPsThreads) dst[i] = src[i];
    };
    if (threadIdx.x == 0) {
        mbar_init(bars, 1u);
        mbar_init(bars + 8u, 1u);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    load_layer(0);
    if (P.n_layers > 1) load_layer(1);
    __syncthreads();
    PsCursor cur;
    ps_issue(P, ring, cur, slots, P.slot_bytes, bars);
    ps_issue(P, ring, cur, slots, P.slot_bytes, bars);
    // embedding row (bit-exact block dequant), spread over the grid
    {
        int t = tok;
        if (t < 0 || t >= P.embd.L.rows) {
            if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&P.st->error, 1u);
            t = 0;
        }
        switch (P.embd.L.type) {
        case kQ8_0: ps_embed<kQ8_0>(P.embd, t, P.h); break;
        case kQ5_0: ps_embed<kQ5_0>(P.embd, t, P.h); break;
        case kQ4_K: ps_embed<kQ4_K>(P.embd, t, P.h); break;
        default: ps_embed<kQ6_K>(P.embd, t, P.h); break;
        }
    }
    unsigned int nbar = 0;
    bool ok = grid_sync(P.bar, ++nbar, P.st);
    const int hd = 64, dim = P.dim, kvd = P.kv_heads * hd;
    const int nchunk = (pos + kAttnChunk) / kAttnChunk;
    int seq = 0;  // sequence number of the next unit to compute
    // one unit: compute from its slot, then reuse the slot for the unit two ahead
    auto unit = [&](const PGemv &g, const float *x, int pre, const float *aux, float *y, const float *add,
                    bool reuse) {
        if (!ok) return;
        ok = ps_gemv_any(g, seq, slots, P.slot_bytes, bars, x, pre, aux, P.eps, y, add, smem, parts, red, P.bar,
                         P.st, reuse);
        ++seq;
        ps_issue(P, ring, cur, slots, P.slot_bytes, bars);
    };
    for (int l = 0; l < P.n_layers && ok; ++l) {
        const PLayer &ly = ring[l & 1];
        // 1: [q; k; v] with the RMSNorm prologue and the biases
        if (ly.n_qkv == 1) {
            unit(ly.qkv[0], P.h, kPreRmsNorm, ly.attn_norm, P.qkv, ly.bias_qkv, false);
        } else {
            const int f0 = slice_family(ly.qkv[0].L.type), f1 = slice_family(ly.qkv[1].L.type);
            unit(ly.qkv[0], P.h, kPreRmsNorm, ly.attn_norm, P.qkv, ly.bias_qkv, false);
            unit(ly.qkv[1], P.h, kPreRmsNorm, ly.attn_norm, P.qkv + dim, ly.bias_qkv + dim, f1 == f0);
            unit(ly.qkv[2], P.h, kPreRmsNorm, ly.attn_norm, P.qkv + dim + kvd, ly.bias_qkv + dim + kvd,
                 slice_family(ly.qkv[2].L.type) == f1);
        }
        ok = ok && grid_sync(P.bar, ++nbar, P.st);
        if (!ok) break;
        // 2: attention items; the last CTA of each kv head merges its chunks
        for (int item = blockIdx.x; item < P.kv_heads * nchunk; item += gridDim.x)
            attention_item<64, false, kPsThreads>(attn, item / nchunk, item % nchunk, P.qkv, P.heads, P.kv_heads,
                                                  ly.kc, ly.vc, P.max_ctx, P.rope_base, P.st, P.part, P.attn_cnt,
                                                  P.att);
        ok = grid_sync(P.bar, ++nbar, P.st);
        // 3: o, residual
        unit(ly.o, P.att, kPreNone, nullptr, P.h, P.h, false);
        ok = ok && grid_sync(P.bar, ++nbar, P.st);
        // 4: [gate; up] with the RMSNorm prologue (one matrix: up lands after gate)
        float *up = ly.n_gu == 1 ? P.gate + P.hid : P.up;
        unit(ly.gu[0], P.h, kPreRmsNorm, ly.ffn_norm, P.gate, nullptr, false);
        if (ly.n_gu == 2)
            unit(ly.gu[1], P.h, kPreRmsNorm, ly.ffn_norm, up, nullptr,
                 slice_family(ly.gu[1].L.type) == slice_family(ly.gu[0].L.type));
        ok = ok && grid_sync(P.bar, ++nbar, P.st);
        // 5: down with the SwiGLU prologue, residual; then the descriptor of
        // layer l + 2 takes ring slot l & 1 (the issue cursor is past layer l)
        if (l + 1 == P.n_layers) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        unit(ly.down, P.gate, kPreSwiGlu, up, P.h, P.h, false);
        if (l + 2 < P.n_layers) load_layer(l + 2);
        if (l + 1 < P.n_layers) ok = ok && grid_sync(P.bar, ++nbar, P.st);
    }
    // Copies still in flight into the slots must land before the CTA exits
    // (bounded waits: after an abort a slot may hold an issued unit).
    while (seq < cur.seq) {
        if (!mbar_wait(bars + 8u * (uint32_t)(seq & 1), (uint32_t)((seq >> 1) & 1))) break;
        ++seq;
    }
}

// ------------------------------------------------- Qwen2 prefill
//
// The reference's layer-first chunked prefill (qwen2_prefill_tokens,
// src/qwen2_architecture.cpp:1550-1729) runs chunks of 8 positions through
// every layer.  A query attends only to keys at or before its own position, so
// the chunk length does not change what is computed: here a chunk is up to
// 1024 positions and its projections are batched matmuls (tensor cores from 32
// positions).  These kernels are the steps between the projections.

// One CTA per position: the token's row of the resident embedding (bit-exact,
// as embed_kernel).  A token outside the vocabulary sets error bit 1.
template <uint32_t FMT>
__global__ void embed_rows_kernel(Layout L, const uint8_t *__restrict__ w, const int *__restrict__ ids,
                                  float *__restrict__ h, unsigned int *err)
{
    constexpr int BE = BlockShape<FMT>::E;
    const int b = blockIdx.x;
    int tok = ids[b];
    if (tok < 0 || tok >= L.rows) {
        if (threadIdx.x == 0) atomicOr(err, 1u);
        tok = 0;
    }
    float *out = h + (size_t)b * L.cols;
    uint8_t raw[BlockShape<FMT>::B];
    for (int blk = threadIdx.x; blk < L.nb; blk += blockDim.x) {
        gather_raw_block(L, w + (uint64_t)tok * L.row_stride, blk, raw);
        for (int i = 0; i < BE; ++i) out[blk * BE + i] = dequant_value<FMT>(raw, i);
    }
}

constexpr int kRowThreads = 256;

// One CTA per row: out = (x / sqrt(mean(x^2) + eps)) * w
// (tensor_rms_norm_f32, src/tensor.cpp:99-136).
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w, float eps, int cols,
                    float *__restrict__ out)
{
    __shared__ float part[kRowThreads / 32];
    const float *xr = x + (size_t)blockIdx.x * cols;
    float *orow = out + (size_t)blockIdx.x * cols;
    float ss = 0.f;
    for (int i = threadIdx.x; i < cols; i += kRowThreads) ss += xr[i] * xr[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < kRowThreads / 32; ++i) ss += part[i];
    const float denom = sqrtf(ss / (float)cols + eps);
    for (int i = threadIdx.x; i < cols; i += kRowThreads) orow[i] = (xr[i] / denom) * w[i];
}

// One CTA per position b (absolute position pos0 + b): the projection biases
// (qwen2_layer_project_batch, :763-807), RoPE on every query and key head
// (transformer_apply_rope_f32, src/transformer_ops.cpp:43-69; q rotated in
// place) and the key/value appended to the layer's cache.
template <int HD>
__global__ void rope_kv_kernel(float *__restrict__ q, int q_ld, const float *__restrict__ k, int k_ld,
                               const float *__restrict__ v, int v_ld, const float *__restrict__ bias_q,
                               const float *__restrict__ bias_k, const float *__restrict__ bias_v, int heads,
                               int kv_heads, int pos0, float rope_base, float *__restrict__ kc,
                               float *__restrict__ vc)
{
    __shared__ float cs[HD / 2], sn[HD / 2];
    const int b = blockIdx.x, pos = pos0 + b, kvd = kv_heads * HD;
    if (threadIdx.x < HD / 2) {
        const float angle = (float)pos / powf(rope_base, (2.0f * (float)threadIdx.x / (float)HD));
        cs[threadIdx.x] = cosf(angle);
        sn[threadIdx.x] = sinf(angle);
    }
    __syncthreads();
    float *qr = q + (size_t)b * q_ld;
    for (int e = threadIdx.x; e < heads * (HD / 2); e += blockDim.x) {
        const int o = (e / (HD / 2)) * HD, i = e % (HD / 2);
        const float x = qr[o + i] + bias_q[o + i], y = qr[o + i + HD / 2] + bias_q[o + i + HD / 2];
        qr[o + i] = x * cs[i] - y * sn[i];
        qr[o + i + HD / 2] = x * sn[i] + y * cs[i];
    }
    const float *kr = k + (size_t)b * k_ld;
    float *kdst = kc + (size_t)pos * kvd;
    for (int e = threadIdx.x; e < kv_heads * (HD / 2); e += blockDim.x) {
        const int o = (e / (HD / 2)) * HD, i = e % (HD / 2);
        const float x = kr[o + i] + bias_k[o + i], y = kr[o + i + HD / 2] + bias_k[o + i + HD / 2];
        kdst[o + i] = x * cs[i] - y * sn[i];
        kdst[o + i + HD / 2] = x * sn[i] + y * cs[i];
    }
    const float *vr = v + (size_t)b * v_ld;
    float *vdst = vc + (size_t)pos * kvd;
    for (int e = threadIdx.x; e < kvd; e += blockDim.x) vdst[e] = vr[e] + bias_v[e];
}

constexpr int kPfKeys = 64;   // keys per shared-memory tile
constexpr int kPfWarps = 8;   // 16 query rows each (one m16 tile)
constexpr int kPfRows = 16 * kPfWarps;
constexpr int kPfPairs = kPfKeys / 2 + 4;  // 32-bit words per smem row: 64 bf16 + 8 of padding
// dynamic shared memory: the raw fp32 K and V rows of the next tile (filled by
// cp.async while the current tile's MMAs run), then the split bf16 planes of
// the current tile
constexpr int kPfRawFloats = kPfKeys * 64;
constexpr size_t kPfSmem = sizeof(float) * 2 * kPfRawFloats + sizeof(uint32_t) * 4 * 64 * kPfPairs;
constexpr int kPfMaxSplits = 8;  // key-range splits per query block (partials per row)

// 16-byte global -> shared copy, L2 only; src_bytes 0 fills zeros (the source
// is then not read).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Packed bf16 hi/lo parts of (a, b): hi = each rounded to 8 significant bits,
// lo = the remainder rounded likewise; a = hi + lo to about 2^-16 relative.
// The element with the lower index sits in the lower half (MMA fragment order).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t &h, uint32_t &l)
{
    const float2 x = f2(a, b);
    const float2 hi = round8x2(x);
    const float2 lo = round8x2(__ffma2_rn(hi, f2(-1.f, -1.f), x));
    h = __byte_perm(__float_as_uint(hi.x), __float_as_uint(hi.y), 0x7632u);
    l = __byte_perm(__float_as_uint(lo.x), __float_as_uint(lo.y), 0x7632u);
}

// d += a b for one 16x8x16 bf16 tile (fp32 accumulate), fragments in the
// mma.sync register layout.
__device__ __forceinline__ void mma_bf16_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// x y to fp32 accuracy from the split parts: xh yh + xl yh + xh yl.
__device__ __forceinline__ void mma_split(float d[4], const uint32_t ah[4], const uint32_t al[4], uint32_t bh0,
                                          uint32_t bh1, uint32_t bl0, uint32_t bl1)
{
    mma_bf16_16816(d, ah, bh0, bh1);
    mma_bf16_16816(d, al, bh0, bh1);
    mma_bf16_16816(d, ah, bl0, bl1);
}

// Key tiles of query block y (positions b0 .. b0 + nq - 1 of the chunk) and
// the number of key-range splits its rows take.
__device__ __forceinline__ int pf_tiles(int pos0, int b0, int nq) { return (pos0 + b0 + nq - 1) / kPfKeys + 1; }

// Causal grouped-query attention for n consecutive positions pos0.. of one
// chunk (transformer_attention_f32, src/transformer_ops.cpp:71-161, over the
// position + 1 keys each query sees, :1640-1648).  Grid (KV head g, block of
// qt positions, key-range split z of tps tiles); a CTA's rows are (position,
// query head of group g), 16 per warp.  A block whose keys span one split
// writes its rows normalised to att; otherwise each split stores its rows'
// (running max, sum of exp, unnormalised output) in part, and the block's
// last split CTA to finish (an arrival counter, re-armed by it) combines them:
// out = sum_z e^(m_z - M) o_z / sum_z e^(m_z - M) l_z, the softmax over all
// of a row's keys.  Keys and values stream through shared memory 64 at a time from the
// layer's cache (which already holds this chunk's keys) as bf16 hi/lo parts;
// Q K^T and P V run on the tensor cores (mma.sync m16n8k16) with three
// products per split pair (dropping only lo x lo, ~2^-16 relative), fp32
// accumulation, and an online softmax in registers: the score tile's
// accumulator layout is the A-fragment layout of P, so scores never leave
// registers.  Scores are divided by sqrt(head_dim) as the reference does.
template <int HD>
__global__ void __launch_bounds__(kPfWarps * 32, 2)
prefill_attention_kernel(const float *__restrict__ q, int q_ld, const float *__restrict__ kc,
                         const float *__restrict__ vc, int heads, int kv_heads, int pos0, int n, int qt, int tps,
                         float *__restrict__ att, float *__restrict__ part, unsigned int *__restrict__ counter)
{
    static_assert(HD == 64, "four 16-wide K steps, eight 8-wide output tiles");
    extern __shared__ __align__(16) float pf_sm[];
    float *raw = pf_sm;  // [K | V][key][d]
    uint32_t(*kh)[kPfPairs] = reinterpret_cast<uint32_t(*)[kPfPairs]>(pf_sm + 2 * kPfRawFloats);  // [key][d pair]
    uint32_t(*kl)[kPfPairs] = kh + kPfKeys;
    uint32_t(*vh)[kPfPairs] = kl + kPfKeys;  // [d][key pair]
    uint32_t(*vl)[kPfPairs] = vh + HD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gr = lane >> 2, tg = lane & 3;
    const int kvh = blockIdx.x, G = heads / kv_heads, kvd = kv_heads * HD, dim = heads * HD;
    const int b0 = blockIdx.y * qt, nq = min(qt, n - b0), rows = nq * G;
    const int ntiles = pf_tiles(pos0, b0, nq), splits = (ntiles + tps - 1) / tps, z = blockIdx.z;
    if (z >= splits) return;
    const int ra = warp * 16 + gr, rb = ra + 8;  // this thread's two rows
    const int pa = ra < rows ? pos0 + b0 + ra / G : -1, pb = rb < rows ? pos0 + b0 + rb / G : -1;
    // Q fragments of both rows for the four 16-wide d steps, split once
    uint32_t qh[4][4], ql[4][4];
    {
        const float *qa = ra < rows ? q + (size_t)(b0 + ra / G) * q_ld + (kvh * G + ra % G) * HD : nullptr;
        const float *qb = rb < rows ? q + (size_t)(b0 + rb / G) * q_ld + (kvh * G + rb % G) * HD : nullptr;
#pragma unroll
        for (int st = 0; st < 4; ++st) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // d = 16 st + 8 half + 2 tg
                const int d = 16 * st + 8 * half + 2 * tg;
                const float2 xa = qa ? *reinterpret_cast<const float2 *>(qa + d) : f2(0.f, 0.f);
                const float2 xb = qb ? *reinterpret_cast<const float2 *>(qb + d) : f2(0.f, 0.f);
                split_pair(xa.x, xa.y, qh[st][2 * half], ql[st][2 * half]);
                split_pair(xb.x, xb.y, qh[st][2 * half + 1], ql[st][2 * half + 1]);
            }
        }
    }
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
    const float rs = sqrtf((float)HD);
    const int last = pos0 + b0 + nq - 1;  // keys [0, last] are visible to some row
    const int tb = z * tps * kPfKeys, te = min((z + 1) * tps * kPfKeys, last + 1);  // this split's keys
    const uint32_t raw_s = (uint32_t)__cvta_generic_to_shared(raw);
    // raw K and V rows of the tile at t0 (keys past `last` are zero-filled,
    // never read)
    auto fetch = [&](int t0) {
        for (int e = tid; e < kPfKeys * (HD / 4); e += kPfWarps * 32) {
            const int key = e / (HD / 4), c4 = e % (HD / 4);
            const bool ok = t0 + key <= last;
            const size_t src = ok ? (size_t)(t0 + key) * kvd + kvh * HD + 4 * c4 : 0;
            const uint32_t dst = raw_s + 4u * (uint32_t)(key * HD + 4 * c4);
            cp_async16(dst, kc + src, ok ? 16u : 0u);
            cp_async16(dst + 4u * kPfRawFloats, vc + src, ok ? 16u : 0u);
        }
        cp_async_commit();
    };
    fetch(tb);
    for (int t0 = tb; t0 < te; t0 += kPfKeys) {
        const int tn = min(kPfKeys, last + 1 - t0);
        cp_async_wait<0>();
        __syncthreads();  // this tile's raw rows are visible; the previous tile's planes are consumed
        const float *kr = raw, *vr = raw + kPfRawFloats;
        for (int e = tid; e < kPfKeys * (HD / 2); e += kPfWarps * 32) {
            const int key = e / (HD / 2), dp = e % (HD / 2);
            const float2 kk = *reinterpret_cast<const float2 *>(kr + key * HD + 2 * dp);
            split_pair(kk.x, kk.y, kh[key][dp], kl[key][dp]);
        }
        for (int e = tid; e < (kPfKeys / 2) * HD; e += kPfWarps * 32) {
            const int kp = e / HD, d = e % HD;
            split_pair(vr[2 * kp * HD + d], vr[(2 * kp + 1) * HD + d], vh[d][kp], vl[d][kp]);
        }
        __syncthreads();                               // planes ready, raw buffer free
        if (t0 + kPfKeys < te) fetch(t0 + kPfKeys);  // in flight during this tile's MMAs
        // S = Q K^T: tile j holds keys t0 + 8 j + 2 tg + {0, 1} of rows ra (0, 1) and rb (2, 3)
        float sc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
            for (int st = 0; st < 4; ++st)
                mma_split(sc[j], qh[st], ql[st], kh[8 * j + gr][8 * st + tg], kh[8 * j + gr][8 * st + 4 + tg],
                          kl[8 * j + gr][8 * st + tg], kl[8 * j + gr][8 * st + 4 + tg]);
        }
        float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int key = t0 + 8 * j + 2 * tg + c;
                sc[j][c] = key - t0 < tn && key <= pa ? sc[j][c] / rs : -INFINITY;
                sc[j][2 + c] = key - t0 < tn && key <= pb ? sc[j][2 + c] / rs : -INFINITY;
                mxa = fmaxf(mxa, sc[j][c]);
                mxb = fmaxf(mxb, sc[j][2 + c]);
            }
        }
#pragma unroll
        for (int off = 1; off < 4; off <<= 1) {  // the four lanes of a row
            mxa = fmaxf(mxa, __shfl_xor_sync(kFull, mxa, off));
            mxb = fmaxf(mxb, __shfl_xor_sync(kFull, mxb, off));
        }
        const float na = fmaxf(ma, mxa), nb = fmaxf(mb, mxb);
        // a row with no visible key yet (a padding row) keeps zero weights
        const float ca = na == -INFINITY ? 1.f : expf(ma - na), cb = nb == -INFINITY ? 1.f : expf(mb - nb);
        la *= ca;
        lb *= cb;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= ca;
            o[j][1] *= ca;
            o[j][2] *= cb;
            o[j][3] *= cb;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                sc[j][c] = na == -INFINITY ? 0.f : expf(sc[j][c] - na);
                sc[j][2 + c] = nb == -INFINITY ? 0.f : expf(sc[j][2 + c] - nb);
                la += sc[j][c];
                lb += sc[j][2 + c];
            }
        }
        ma = na;
        mb = nb;
        // O += P V: the k-step st (keys 16 st ..) takes P from score tiles 2 st, 2 st + 1
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            uint32_t ph[4], pl[4];
            split_pair(sc[2 * st][0], sc[2 * st][1], ph[0], pl[0]);
            split_pair(sc[2 * st][2], sc[2 * st][3], ph[1], pl[1]);
            split_pair(sc[2 * st + 1][0], sc[2 * st + 1][1], ph[2], pl[2]);
            split_pair(sc[2 * st + 1][2], sc[2 * st + 1][3], ph[3], pl[3]);
#pragma unroll
            for (int jd = 0; jd < 8; ++jd)
                mma_split(o[jd], ph, pl, vh[8 * jd + gr][8 * st + tg], vh[8 * jd + gr][8 * st + 4 + tg],
                          vl[8 * jd + gr][8 * st + tg], vl[8 * jd + gr][8 * st + 4 + tg]);
        }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        la += __shfl_xor_sync(kFull, la, off);
        lb += __shfl_xor_sync(kFull, lb, off);
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int r = h2 ? rb : ra;
        if (r >= rows) continue;
        const float l = h2 ? lb : la, mm = h2 ? mb : ma;
        const int b = b0 + r / G, head = kvh * G + r % G;
        if (splits == 1) {
            float *out = att + (size_t)b * dim + head * HD;
#pragma unroll
            for (int jd = 0; jd < 8; ++jd)
                *reinterpret_cast<float2 *>(out + 8 * jd + 2 * tg) = f2(o[jd][2 * h2] / l, o[jd][2 * h2 + 1] / l);
        } else {
            float *pp = part + ((size_t)(b * heads + head) * kPfMaxSplits + z) * (HD + 2);
            if (tg == 0) {
                pp[0] = mm;
                pp[1] = l;
            }
#pragma unroll
            for (int jd = 0; jd < 8; ++jd) {
                pp[2 + 8 * jd + 2 * tg] = o[jd][2 * h2];
                pp[3 + 8 * jd + 2 * tg] = o[jd][2 * h2 + 1];
            }
        }
    }
    if (splits == 1) return;
    // the last split CTA of this block merges every split's rows
    __shared__ int last_cta;
    __threadfence();
    __syncthreads();
    unsigned int *cnt = counter + (size_t)kvh * gridDim.y + blockIdx.y;
    if (tid == 0) last_cta = atomicAdd(cnt, 1u) == (unsigned)(splits - 1);
    __syncthreads();
    if (!last_cta) return;
    __threadfence();
    float *wgt = reinterpret_cast<float *>(&kh[0][0]);  // [row][split] weights, then 1 / denominator per row
    float *inv = wgt + kPfRows * kPfMaxSplits;
    for (int r = tid; r < rows; r += kPfWarps * 32) {
        const float *pp = part + (size_t)((b0 + r / G) * heads + kvh * G + r % G) * kPfMaxSplits * (HD + 2);
        float M = -INFINITY;
        for (int zz = 0; zz < splits; ++zz) M = fmaxf(M, pp[zz * (HD + 2)]);
        float den = 0.f;
        for (int zz = 0; zz < splits; ++zz) {
            const float mz = pp[zz * (HD + 2)];
            const float wz = mz == -INFINITY ? 0.f : expf(mz - M);
            wgt[r * kPfMaxSplits + zz] = wz;
            den += wz * pp[zz * (HD + 2) + 1];
        }
        inv[r] = den;
    }
    __syncthreads();
    // two output columns per thread and step, every split's loads issued together
#pragma unroll 2
    for (int e = tid; e < rows * (HD / 2); e += kPfWarps * 32) {
        const int r = e / (HD / 2), d = 2 * (e % (HD / 2)), b = b0 + r / G, head = kvh * G + r % G;
        const float *pp = part + (size_t)(b * heads + head) * kPfMaxSplits * (HD + 2) + 2 + d;
        float2 v[kPfMaxSplits];
#pragma unroll
        for (int zz = 0; zz < kPfMaxSplits; ++zz)
            v[zz] = zz < splits ? *reinterpret_cast<const float2 *>(pp + zz * (HD + 2)) : f2(0.f, 0.f);
        float n0 = 0.f, n1 = 0.f;
#pragma unroll
        for (int zz = 0; zz < kPfMaxSplits; ++zz) {
            const float wz = zz < splits ? wgt[r * kPfMaxSplits + zz] : 0.f;
            n0 += wz * v[zz].x;
            n1 += wz * v[zz].y;
        }
        *reinterpret_cast<float2 *>(att + (size_t)b * dim + head * HD + d) = f2(n0 / inv[r], n1 / inv[r]);
    }
    if (tid == 0) *cnt = 0u;
}

// out = up * silu(gate) row by row (transformer_swiglu_f32,
// src/transformer_ops.cpp:163-178); gate and up may be the halves of one
// [gate | up] row.
__global__ void swiglu_rows_kernel(const float *__restrict__ gate, int g_ld, const float *__restrict__ up, int u_ld,
                                   int cols, int rows, float *__restrict__ out)
{
    const size_t n = (size_t)rows * cols;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const size_t r = e / cols, c = e % cols;
        const float x = gate[r * g_ld + c];
        out[e] = up[r * u_ld + c] * (x / (1.0f + expf(-x)));
    }
}

// ------------------------------------------------------ launch helpers

// The calling thread's own status word for the launches it makes (set around
// the drop-in calls; null otherwise).
thread_local unsigned int *t_call_status = nullptr;

int sm_count()
{
    static int count = 0;
    if (count == 0) {
        int dev = 0, n = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        count = n > 0 ? n : 148;
    }
    return count;
}

unsigned grid_for(uint64_t work, int threads)
{
    uint64_t g = (work + threads - 1) / threads;
    uint64_t cap = (uint64_t)sm_count() * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (unsigned)g;
}

// The dynamic shared-memory limit is per-function state: raise it once per
// (kernel, device) to the opt-in maximum, so a later launch with less shared
// memory never lowers it below what another shape needs.
cudaError_t allow_max_smem(const void *fn, int dev)
{
    struct Entry {
        const void *fn;
        int dev;
    };
    static thread_local Entry done[64];
    static thread_local int used = 0;
    for (int i = 0; i < used; ++i)
        if (done[i].fn == fn && done[i].dev == dev) return cudaSuccess;
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes attr;
    e = cudaFuncGetAttributes(&attr, fn);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)attr.sharedSizeBytes);
    if (e != cudaSuccess) return e;
    if (used < 64) done[used++] = Entry{fn, dev};
    return cudaSuccess;
}

// Per-thread cache of (device, kernel, shared bytes) -> resident CTAs per SM.
template <typename K>
cudaError_t prepare(K kernel, size_t smem, int *blocks_per_sm)
{
    struct Entry {
        const void *fn;
        int dev;
        size_t smem;
        int occ;
    };
    static thread_local Entry cache[64];
    static thread_local int used = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    for (int i = 0; i < used; ++i) {
        if (cache[i].fn == (const void *)kernel && cache[i].dev == dev && cache[i].smem == smem) {
            *blocks_per_sm = cache[i].occ;
            return cudaSuccess;
        }
    }
    e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (*blocks_per_sm < 1) return cudaErrorInvalidConfiguration;
    if (used < 64) cache[used++] = Entry{(const void *)kernel, dev, smem, *blocks_per_sm};
    return cudaSuccess;
}

template <uint32_t FMT, int TPT, int R>
cudaError_t gemv_go(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut *am,
                    cudaStream_t s)
{
    auto kernel = gemv_kernel<FMT, TPT, R>;
    const size_t smem = xs_bytes(L.cols);
    int occ = 0;
    cudaError_t e = prepare(kernel, smem, &occ);
    if (e != cudaSuccess) return e;
    constexpr int WR = (32 / TPT) * R;
    const long long warp_tiles = ((long long)L.rows + WR - 1) / WR;
    long long grid = (long long)sm_count() * occ;
    const long long useful = (warp_tiles + (kThreads / 32) - 1) / (kThreads / 32);
    if (grid > useful) grid = useful;
    if (am && grid > kMaxArgmaxCtas) grid = kMaxArgmaxCtas;
    if (grid < 1) grid = 1;
    ArgmaxOut a = am ? *am : ArgmaxOut{nullptr, nullptr, 0};
    kernel<<<(unsigned)grid, kThreads, smem, s>>>(L, w, x, y, a, am ? 1 : 0);
    return cudaGetLastError();
}

// 0 auto (resident-row-range kernel, else exclusive TMA plan, else direct
// loads), 1 direct loads, 2 TMA pipeline only, 3 exclusive TMA plan (else
// direct loads), 4 the shared TMA plan where it fits (else as 3), 5 the
// resident-row-range kernel only
int g_gemv_path = 0;

// Decode attention: 0 the cluster kernel where the group has at most 8 query
// heads and the device can place a 16-CTA cluster, 1 the chunked kernel.
int g_attn_path = 0;

// Whether a 16-CTA cluster of attention_cluster_kernel fits on the current
// device (non-portable cluster size; checked once per device).
bool attention_cluster_ok()
{
    static std::mutex mu;
    static int state[64] = {};  // 0 unknown, 1 yes, 2 no
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (state[dev] == 0) {
        bool ok = cudaFuncSetAttribute(attention_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                      cudaSuccess &&
                  cudaFuncSetAttribute(attention_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kDaSmem) == cudaSuccess;
        if (ok) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(kDaSplit);
            cfg.blockDim = dim3(kDaThreads);
            cfg.dynamicSmemBytes = kDaSmem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = kDaSplit;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int clusters = 0;
            ok = cudaOccupancyMaxActiveClusters(&clusters, attention_cluster_kernel, &cfg) == cudaSuccess &&
                 clusters > 0;
        }
        cudaGetLastError();  // a refused attribute is not an error of a later call
        state[dev] = ok ? 1 : 2;
    }
    return state[dev] == 1;
}

// Shared-memory plan of the TMA kernel: the first of these (consumer warps,
// rows per warp, minimum stages) whose stages fit.  Two rows per warp share
// each x slice load, so they come first; 16 warps hide shared-memory latency
// better than 8.  batched: the plan of the batched kernel (np positions of
// x in shared memory, 8 consumer warps).  false when none fits (the
// direct-load kernels run).
constexpr uint32_t kTmaBudget = 227u * 1024u - 2048u;  // dynamic bytes, leaving room for the static ~1.6 KB
// Two CTAs per SM: each takes at most half of the SM's 228 KiB, less its
// static shared memory (~1.6 KB) and the 1 KiB the system reserves per CTA.
constexpr uint32_t kTmaBudgetShared = 111u * 1024u;

// One candidate {consumer warps, rows per warp, minimum stages, warps per
// row} for a matrix whose rows spread over ctas CTAs; false when its stages
// do not fit.
bool tma_candidate(const Layout &L, const int *cand, int np, long long ctas, TmaPlan *P, uint32_t budget)
{
    const uint32_t xb = (uint32_t)((xs_bytes(L.cols) * (size_t)np + 127) & ~(size_t)127);
    if (xb >= budget || ctas < 1) return false;
    const int cw = cand[0], r = cand[1], min_stages = cand[2], split = cand[3];
    const uint64_t sb = ((uint64_t)cw * r / split * L.row_stride + 127) & ~127ull;
    const uint64_t ns = (budget - xb) / sb;
    if ((int)ns < min_stages) return false;
    P->x_bytes = xb;
    P->stage_bytes = (uint32_t)sb;
    P->rows_per_stage = cw * r / split;
    // no more stages than one CTA's rows fill, at least 2: small matrices then
    // leave shared memory for the CTAs of the launches around them
    const long long per_cta = ((long long)L.rows + ctas - 1) / ctas;
    const long long need = (per_cta + P->rows_per_stage - 1) / P->rows_per_stage;
    uint64_t cap = need < 2 ? 2 : (uint64_t)need;
    if (cap > 8) cap = 8;
    P->stages = (int)(ns > cap ? cap : ns);
    P->consumer_warps = cw;
    P->rows_per_warp = r;
    P->np = np;
    P->split = split;
    P->status = nullptr;
    return true;
}

bool tma_plan(const Layout &L, TmaPlan *P, int np = 1, bool batched = false)
{
    static const int kCandidates[][4] = {{16, 2, 2, 1}, {8, 2, 3, 1}, {16, 1, 3, 1}, {8, 2, 2, 1},
                                         {16, 1, 2, 1}, {16, 1, 2, 2}, {8, 1, 2, 1}};
    // batched form: 8 warps of two rows (each x slice load serves two rows;
    // 16 warps of one row measured slower on configuration 3 at 8 positions,
    // 9.2 vs 8.3 us)
    static const int kBatchCandidates[][4] = {{8, 2, 2, 1}, {8, 1, 2, 1}};
    const long long ctas = L.rows < sm_count() ? L.rows : sm_count();  // one CTA per SM
    // Short rows (one 32-lane pass per row) with many rows per CTA: 8 warps
    // of four rows, so a stage's wait, reductions and epilogue serve four
    // rows (the Q8_0 151936 x 896 output projection: 33.3 -> 26.6 us).
    static const int kShortRows[][4] = {{8, 4, 3, 1}, {8, 4, 2, 1}};
    if (!batched && L.C <= 32 && (long long)L.rows >= 64 * ctas)
        for (const int *cand : kShortRows)
            if (tma_candidate(L, cand, np, ctas, P, kTmaBudget)) return true;
    const int n_cand = batched ? 2 : 7;
    for (int ci = 0; ci < n_cand; ++ci)
        if (tma_candidate(L, batched ? kBatchCandidates[ci] : kCandidates[ci], np, ctas, P, kTmaBudget))
            return true;
    return false;
}

// The shared plan: one CTA per SM whose stages fit in half of the SM's shared
// memory (and whose kernel instance is capped to half the registers), so the
// CTA of the next launch in the stream can be resident beside it and stream
// its first stages while this one computes its last.  Single position, no
// split rows.
bool tma_plan_shared(const Layout &L, TmaPlan *P)
{
    static const int kShared[][4] = {{16, 2, 2, 1}, {16, 1, 3, 1}, {8, 2, 3, 1}, {16, 1, 2, 1}, {8, 2, 2, 1}};
    const long long ctas = L.rows < sm_count() ? L.rows : sm_count();
    for (const int *cand : kShared)
        if (tma_candidate(L, cand, 1, ctas, P, kTmaBudgetShared)) return true;
    return false;
}

// Plan of the resident-row-range kernel for one matrix, or two with equal
// columns sharing x: one CTA per SM (fewer for fewer rows); false when a
// CTA's rows or the quantized x exceed their budgets.
bool lite_plan(const LiteMat *mats, int n, LitePlan *P, unsigned *grid_out)
{
    long long grid = sm_count();
    for (int i = 0; i < n; ++i)
        if (grid > mats[i].L.rows) grid = mats[i].L.rows;
    if (grid < 1) return false;
    const uint32_t xb = (uint32_t)((xs_bytes(mats[0].L.cols) + 127) & ~(size_t)127);
    if (xb > kLiteXBudget) return false;
    uint64_t off = 0;
    for (int i = 0; i < n; ++i) {
        const uint64_t max_rows = ((uint64_t)mats[i].L.rows + (uint64_t)grid - 1) / (uint64_t)grid;
        P->m[i] = mats[i];
        P->m[i].soff = (uint32_t)off;
        off += (max_rows * mats[i].L.row_stride + 127) & ~127ull;
        if (off > kLiteRowBudget) return false;
    }
    P->nmat = n;
    P->x_bytes = xb;
    P->smem = xb + (uint32_t)off;
    if (P->smem < kLiteSmemFloor) P->smem = kLiteSmemFloor;  // at most two CTAs per SM
    P->status = nullptr;
    *grid_out = (unsigned)grid;
    return true;
}

template <uint32_t FA, uint32_t FB, int R>
cudaError_t gemv_lite_go_r(const LitePlan &P, unsigned grid, const float *x, const ArgmaxOut *am, const Fuse &fu,
                           cudaStream_t s)
{
    auto kernel = gemv_lite_kernel<FA, FB, R>;
    LitePlan Pc = P;
    Pc.status = t_call_status;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    const ArgmaxOut a = am ? *am : ArgmaxOut{nullptr, nullptr, 0};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kLiteWarps * 32);
    cfg.dynamicSmemBytes = P.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, Pc, x, a, am ? 1 : 0, fu);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// One row per warp pass when a CTA holds at most one row per warp (all warps
// busy), else two (each x slice load serves two rows).
template <uint32_t FA, uint32_t FB>
cudaError_t gemv_lite_go(const LitePlan &P, unsigned grid, const float *x, const ArgmaxOut *am, const Fuse &fu,
                         cudaStream_t s)
{
    const int per_cta = (P.m[0].L.rows + (int)grid - 1) / (int)grid;
    if (per_cta <= kLiteWarps) return gemv_lite_go_r<FA, FB, 1>(P, grid, x, am, fu, s);
    return gemv_lite_go_r<FA, FB, 2>(P, grid, x, am, fu, s);
}

// One matrix on the resident-row-range kernel under the current path
// setting (automatic or forced); cudaErrorNotSupported when it does not
// apply.
template <uint32_t FMT>
cudaError_t gemv_lite_single(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut *am,
                             const Fuse &fu, cudaStream_t s)
{
    if (g_gemv_path != 0 && g_gemv_path != 5) return cudaErrorNotSupported;
    const LiteMat m{L, w, y, fu.add, 0};
    LitePlan P;
    unsigned grid = 0;
    if (!lite_plan(&m, 1, &P, &grid)) return g_gemv_path == 5 ? cudaErrorInvalidConfiguration : cudaErrorNotSupported;
    return gemv_lite_go<FMT, 0>(P, grid, x, am, fu, s);
}

// Plan of a single-position GEMV under the current path setting; *shared
// tells which kernel instance the plan is for.  The exclusive plan is the
// default: measured on B200, the shared plan (register-capped, half the
// stages) cost more in the consumers than the overlap of neighbouring
// launches saved, except on the smallest matrices.
bool gemv_plan(const Layout &L, TmaPlan *P, bool *shared)
{
    *shared = false;
    if (g_gemv_path == 4 && tma_plan_shared(L, P)) {
        *shared = true;
        return true;
    }
    return tma_plan(L, P);
}

template <uint32_t FMT, int CW, int R, int NP = 1, int SPLIT = 1, int MINB = 1>
cudaError_t gemv_tma_go(const Layout &L, const TmaPlan &P, const uint8_t *w, const float *x, float *y,
                        const ArgmaxOut *am, cudaStream_t s, const Exchange &ex = Exchange{},
                        const Fuse &fu = Fuse{})
{
    auto kernel = gemv_tma_kernel<FMT, CW, R, NP, SPLIT, MINB>;
    TmaPlan Pc = P;
    Pc.status = t_call_status;
    const size_t smem = (size_t)P.x_bytes + (size_t)P.stages * P.stage_bytes;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    long long grid = sm_count();
    // the exchange: every rank launches the same number of CTAs (min(SMs,
    // slot rows)); ranks with fewer rows have CTAs without rows
    const long long rows_for_grid = ex.world > 1 ? ex.slot_rows : L.rows;
    if (grid > rows_for_grid) grid = rows_for_grid;
    if (ex.world > 1 && grid > kMaxExCtas) grid = kMaxExCtas;
    Exchange exc = ex;
    exc.ncta = (int)grid;
    ArgmaxOut a = am ? *am : ArgmaxOut{nullptr, nullptr, 0};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((CW + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int want = am ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kernel, L, w, x, y, a, want, Pc, exc, fu);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Launch the single-position TMA GEMV instance that plan P was made for
// (shared: the register-capped instance; 8-warp CTAs fit twice per SM
// without a cap).
template <uint32_t FMT>
cudaError_t gemv_tma_dispatch(const Layout &L, const TmaPlan &P, bool shared, const uint8_t *w, const float *x,
                              float *y, const ArgmaxOut *am, cudaStream_t s, const Exchange &ex = Exchange{},
                              const Fuse &fu = Fuse{})
{
    if (P.split == 2) return gemv_tma_go<FMT, 16, 1, 1, 2>(L, P, w, x, y, am, s, ex, fu);
    if (P.consumer_warps == 16) {
        if (shared)
            return P.rows_per_warp == 2 ? gemv_tma_go<FMT, 16, 2, 1, 1, 2>(L, P, w, x, y, am, s, ex, fu)
                                        : gemv_tma_go<FMT, 16, 1, 1, 1, 2>(L, P, w, x, y, am, s, ex, fu);
        return P.rows_per_warp == 2 ? gemv_tma_go<FMT, 16, 2>(L, P, w, x, y, am, s, ex, fu)
                                    : gemv_tma_go<FMT, 16, 1>(L, P, w, x, y, am, s, ex, fu);
    }
    if (P.rows_per_warp == 4) return gemv_tma_go<FMT, 8, 4>(L, P, w, x, y, am, s, ex, fu);
    return P.rows_per_warp == 2 ? gemv_tma_go<FMT, 8, 2>(L, P, w, x, y, am, s, ex, fu)
                                : gemv_tma_go<FMT, 8, 1>(L, P, w, x, y, am, s, ex, fu);
}

template <uint32_t FMT>
cudaError_t gemv_exchange_fmt(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut &am,
                              const Exchange &ex, cudaStream_t s)
{
    TmaPlan P;
    if (!tma_plan(L, &P)) return cudaErrorNotSupported;
    return gemv_tma_dispatch<FMT>(L, P, false, w, x, y, &am, s, ex);
}

template <uint32_t FMT>
cudaError_t gemv_fused_fmt(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut *am,
                           const Fuse &fu, cudaStream_t s)
{
    // The decode step's fused projections keep the TMA pipeline unless the
    // resident-row-range kernel is forced: in that chain its launches follow
    // attention CTAs that leave some SMs empty early, the next launch then
    // doubles up on those SMs, and the step measured slower (822 vs 683 us
    // per configuration-4 token on B200).
    const cudaError_t el =
        g_gemv_path == 5 ? gemv_lite_single<FMT>(L, w, x, y, am, fu, s) : cudaErrorNotSupported;
    if (el != cudaErrorNotSupported) return el;
    TmaPlan P;
    bool shared = false;
    if (!gemv_plan(L, &P, &shared)) return cudaErrorNotSupported;
    return gemv_tma_dispatch<FMT>(L, P, shared, w, x, y, am, s, Exchange{}, fu);
}

template <uint32_t FA, uint32_t FB, int R>
cudaError_t gemv_pair_go(const GemvPair &pr, int grid, const float *x, const Fuse &fu, cudaStream_t s)
{
    auto kernel = gemv_pair_kernel<FA, FB, 16, R>;
    size_t smem = 0;
    for (int i = 0; i < 2; ++i) {
        const size_t b = (size_t)pr.P[i].x_bytes + (size_t)pr.P[i].stages * pr.P[i].stage_bytes;
        if (b > smem) smem = b;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    GemvPair pc = pr;
    pc.P[0].status = pc.P[1].status = t_call_status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(17 * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, pc, x, fu);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Both matrices take the same 16-warp shape (one block size per launch).
template <uint32_t FA, uint32_t FB>
cudaError_t gemv_pair_fmt(GemvPair pr, int grid, const float *x, const Fuse &fu, cudaStream_t s)
{
    static const int kPairCandidates[][4] = {{16, 2, 2, 1}, {16, 1, 3, 1}, {16, 1, 2, 1}};
    for (const int *cand : kPairCandidates) {
        if (!tma_candidate(pr.L[0], cand, 1, pr.ctas0, &pr.P[0], kTmaBudget) ||
            !tma_candidate(pr.L[1], cand, 1, grid - pr.ctas0, &pr.P[1], kTmaBudget))
            continue;
        return cand[1] == 2 ? gemv_pair_go<FA, FB, 2>(pr, grid, x, fu, s) : gemv_pair_go<FA, FB, 1>(pr, grid, x, fu, s);
    }
    return cudaErrorNotSupported;
}

template <uint32_t FMT>
cudaError_t gemv_fmt(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut *am,
                     cudaStream_t s)
{
    const cudaError_t el = gemv_lite_single<FMT>(L, w, x, y, am, Fuse{}, s);
    if (el != cudaErrorNotSupported) return el;
    TmaPlan P;
    bool shared = false;
    if (g_gemv_path != 1 && gemv_plan(L, &P, &shared)) return gemv_tma_dispatch<FMT>(L, P, shared, w, x, y, am, s);
    if (g_gemv_path == 2) return cudaErrorInvalidConfiguration;
    // 16-lane groups for short rows, whole warps otherwise; two rows per group
    // share each x slice load.
    if (L.C <= 16) return gemv_go<FMT, 16, 2>(L, w, x, y, am, s);
    return gemv_go<FMT, 32, 2>(L, w, x, y, am, s);
}

// Stream-ordered pool for the per-call scratch of the matmul paths (quantized
// or split x), one per device, created on first use.  It keeps freed memory (release
// threshold: unlimited), so steady-state calls allocate without the driver.
cudaError_t scratch_pool(cudaMemPool_t *out)
{
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (pools[dev] == nullptr) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t p = nullptr;
        e = cudaMemPoolCreate(&p, &props);
        if (e != cudaSuccess) return e;
        uint64_t keep = ~0ull;
        e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
        if (e != cudaSuccess) {
            cudaMemPoolDestroy(p);
            return e;
        }
        pools[dev] = p;
    }
    *out = pools[dev];
    return cudaSuccess;
}

}  // namespace

cudaError_t stream_alloc(void **ptr, size_t bytes, cudaStream_t s)
{
    cudaMemPool_t pool;
    const cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    return cudaMallocFromPoolAsync(ptr, bytes, pool, s);
}

cudaError_t stream_free(void *ptr, cudaStream_t s) { return ptr ? cudaFreeAsync(ptr, s) : cudaSuccess; }

namespace {

template <uint32_t FMT, int TPT>
cudaError_t matmul_go(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                      cudaStream_t s)
{
    constexpr int NP = 8;
    auto kernel = matmul_kernel<FMT, TPT, NP>;
    const size_t xb = xs_bytes(L.cols);
    // positions per launch: up to 8, bounded by shared memory (<= 200 KiB)
    int np_max = (int)((200u * 1024u) / xb);
    if (np_max > NP) np_max = NP;
    if (np_max < 1) return cudaErrorInvalidValue;
    int occ = 0;
    cudaError_t e = prepare(kernel, xb * np_max, &occ);
    if (e != cudaSuccess) return e;
    constexpr int GPW = 32 / TPT;
    const long long tiles = ((long long)L.rows + GPW - 1) / GPW;
    long long grid = (long long)sm_count() * occ;
    const long long useful = (tiles + (kThreads / 32) - 1) / (kThreads / 32);
    if (grid > useful) grid = useful;
    if (grid < 1) grid = 1;
    cudaMemPool_t pool;
    e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    void *xq = nullptr;
    e = cudaMallocFromPoolAsync(&xq, (size_t)batch * xb, pool, s);
    if (e != cudaSuccess) return e;
    quantize_x_kernel<FMT><<<(unsigned)batch, kThreads, 0, s>>>(X, L.cols, L.C, (uint8_t *)xq, xb);
    e = cudaGetLastError();
    for (int p0 = 0; p0 < batch && e == cudaSuccess; p0 += np_max) {
        const int np = batch - p0 < np_max ? batch - p0 : np_max;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = xb * np;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, L, w, (const uint8_t *)xq + (size_t)p0 * xb, np,
                               Y + (size_t)p0 * L.rows);
    }
    const cudaError_t f = cudaFreeAsync(xq, s);
    return e != cudaSuccess ? e : f;
}

// 0 auto, 1 CUDA cores (dp4a), 2 tensor cores, 64/128/176/256 tensor cores
// with that position-tile width
int g_matmul_path = 0;

// Batches of at least this many positions take the tensor-core kernel.
constexpr int kTcMinBatch = 32;

template <uint32_t FMT, int TN>
cudaError_t matmul_tc_go(const Layout &L, const uint8_t *w, const XSource &X, int batch, float *Y,
                         cudaStream_t s, int ksplit = 1)
{
    // weight tile in shared memory when it leaves room for at least 3 x stages
    const uint32_t tile_max = (uint32_t)kTcM * (uint32_t)L.row_stride;
    // (a split CTA reads only its columns: it decodes from global memory)
    const bool wsmem = ksplit == 1 && (uint64_t)kTcM * L.row_stride + 3u * tc_stage_bytes(TN) <= kTcSmemBudget;
    int S = wsmem ? (int)((kTcSmemBudget - tile_max) / tc_stage_bytes(TN)) : tc_stages(TN);
    if (S > kTcMaxStages) S = kTcMaxStages;
    auto kernel = wsmem ? matmul_tc_kernel<FMT, TN, true> : matmul_tc_kernel<FMT, TN, false>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    const int n_pt = (batch + TN - 1) / TN, nk = (L.cols + kTcK - 1) / kTcK;
    if (ksplit < 1 || ksplit > nk) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((L.rows + kTcM - 1) / kTcM), (unsigned)n_pt, (unsigned)ksplit);
    if (grid.y > 65535u) return cudaErrorInvalidConfiguration;
    const size_t bytes = (size_t)n_pt * nk * tc_stage_bytes(TN);
    cudaMemPool_t pool;
    e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    void *xs = nullptr;
    e = cudaMallocFromPoolAsync(&xs, bytes, pool, s);
    if (e != cudaSuccess) return e;
    {
        const unsigned g = grid_for((uint64_t)n_pt * nk * TN * (kTcK / 8), kThreads);
        split_x_kernel<TN><<<g, kThreads, 0, s>>>(X, batch, L.cols, nk, (uint8_t *)xs);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        // at least 120 KiB so that one CTA holds an SM (and all of its
        // tensor memory): a second CTA's allocation would wait for the first
        size_t smem = (size_t)S * tc_stage_bytes(TN) + (wsmem ? tile_max : 0u);
        if (smem < 120u * 1024u) smem = 120u * 1024u;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kTcThreads + 64);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, L, w, X, (const uint8_t *)xs, batch, Y, S, t_call_status);
    }
    const cudaError_t f = cudaFreeAsync(xs, s);
    return e != cudaSuccess ? e : f;
}

// Position-tile width of the tensor-core kernel: the candidate with the
// smallest (waves of one-CTA-per-SM tiles) x (per-stage cost), where a
// 64-wide K stage costs max(decode of 128 x 64 weights, 12 MMAs of
// 128 x TN x 16), in SM cycles.
int tc_tile_width(int rows, int batch)
{
    static const int cand[] = {64, 128, 176, 256};
    const long long row_tiles = (rows + kTcM - 1) / kTcM;
    int best = 64;
    double best_cost = 1e300;
    for (int tn : cand) {
        const long long tiles = row_tiles * ((batch + tn - 1) / tn);
        const long long waves = (tiles + sm_count() - 1) / sm_count();
        const double alu = 900.0, mma = 8.4 * tn;
        const double cost = (double)waves * (alu > mma ? alu : mma);
        if (cost < best_cost) {
            best_cost = cost;
            best = tn;
        }
    }
    return best;
}

// Batched form on the int8 tensor cores (Q8_0, Q5_0; chunks of up to 8
// positions) where a CTA's rows (at most 64) and the positions' quantized x
// fit in shared memory; false in *done when it does not apply.
template <uint32_t FMT>
cudaError_t matmul_mma_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y, cudaStream_t s,
                           bool *done)
{
    constexpr int NP = 8;
    *done = false;
    if constexpr (FMT != kQ8_0 && FMT != kQ5_0) {
        return cudaSuccess;
    } else {
        const long long sms = sm_count();
        const long long grid = L.rows < sms ? L.rows : sms;
        const long long per_cta = (L.rows + grid - 1) / grid;
        if (grid < 1 || per_cta > 16 * kMmaMaxTiles) return cudaSuccess;
        const int np0 = batch < NP ? batch : NP;
        const uint32_t xb = (uint32_t)((xs_bytes(L.cols) * (size_t)np0 + 127) & ~(size_t)127);
        const uint64_t rows_bytes = (uint64_t)per_cta * L.row_stride;
        if (xb > 64u * 1024u || rows_bytes > 96u * 1024u) return cudaSuccess;
        const size_t smem = (size_t)xb + rows_bytes;
        auto kernel = matmul_mma_kernel<FMT>;
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        e = allow_max_smem((const void *)kernel, dev);
        if (e != cudaSuccess) return e;
        *done = true;
        for (int p0 = 0; p0 < batch; p0 += NP) {
            const int np = batch - p0 < NP ? batch - p0 : NP;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)grid);
            cfg.blockDim = dim3(kMmaWarps * 32);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaLaunchKernelEx(&cfg, kernel, L, w, X + (size_t)p0 * L.cols, np, Y + (size_t)p0 * L.rows, xb,
                                   t_call_status);
            if (e != cudaSuccess) return e;
        }
        return cudaGetLastError();
    }
}

// Batched CUDA-core form on the TMA pipeline: chunks of up to 8 positions.
// false in *done when no stage plan fits (very long rows).
template <uint32_t FMT>
cudaError_t matmul_tma_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                           cudaStream_t s, bool *done)
{
    constexpr int NP = 8;
    *done = false;
    TmaPlan P;
    if (!tma_plan(L, &P, batch < NP ? batch : NP, true)) return cudaSuccess;
    *done = true;
    for (int p0 = 0; p0 < batch; p0 += NP) {
        const int np = batch - p0 < NP ? batch - p0 : NP;
        if (!tma_plan(L, &P, np, true)) return cudaErrorInvalidConfiguration;
        const float *x = X + (size_t)p0 * L.cols;
        float *y = Y + (size_t)p0 * L.rows;
        const cudaError_t e = P.consumer_warps == 16 ? gemv_tma_go<FMT, 16, 1, NP>(L, P, w, x, y, nullptr, s)
                              : P.rows_per_warp == 2 ? gemv_tma_go<FMT, 8, 2, NP>(L, P, w, x, y, nullptr, s)
                                                     : gemv_tma_go<FMT, 8, 1, NP>(L, P, w, x, y, nullptr, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <uint32_t FMT>
cudaError_t matmul_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                       cudaStream_t s)
{
    // the tensor-core kernel reads x with 16-byte loads
    const bool tc_ok = ((uintptr_t)X & 15u) == 0;
    if (g_matmul_path >= 2 || (g_matmul_path == 0 && batch >= kTcMinBatch && tc_ok)) {
        if (!tc_ok) return cudaErrorMisalignedAddress;
        switch (g_matmul_path > 2 ? g_matmul_path : tc_tile_width(L.rows, batch)) {
        case 64: return matmul_tc_go<FMT, 64>(L, w, XSource{X, nullptr, L.cols, 0}, batch, Y, s);
        case 128: return matmul_tc_go<FMT, 128>(L, w, XSource{X, nullptr, L.cols, 0}, batch, Y, s);
        case 176: return matmul_tc_go<FMT, 176>(L, w, XSource{X, nullptr, L.cols, 0}, batch, Y, s);
        default: return matmul_tc_go<FMT, 256>(L, w, XSource{X, nullptr, L.cols, 0}, batch, Y, s);
        }
    }
    bool done = false;
    if (g_matmul_path == 0) {
        const cudaError_t em = matmul_mma_fmt<FMT>(L, w, X, batch, Y, s, &done);
        if (done || em != cudaSuccess) return em;
    }
    const cudaError_t e = matmul_tma_fmt<FMT>(L, w, X, batch, Y, s, &done);
    if (done || e != cudaSuccess) return e;
    if (L.C <= 16) return matmul_go<FMT, 16>(L, w, X, batch, Y, s);
    return matmul_go<FMT, 32>(L, w, X, batch, Y, s);
}

// out += sum of ks partial slices of n floats (in slice order)
__global__ void add_partials_kernel(float *__restrict__ out, const float *__restrict__ part, size_t n, int ks)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float acc = part[i];
        for (int z = 1; z < ks; ++z) acc += part[(size_t)z * n + i];
        out[i] += acc;
    }
}

constexpr int kTcMaxSplit = 8;

// Tile width and K split of the tensor-core kernel for a residual product:
// the smallest (waves) x ((stages per CTA) x (per-stage cost) + a CTA's
// prologue and epilogue) over the tile widths and splits (one CTA per SM),
// fewer splits on ties.
void tc_split_plan(int rows, int batch, int nk, int *tn_out, int *ks_out)
{
    static const int cand[] = {64, 128, 176, 256};
    const long long row_tiles = (rows + kTcM - 1) / kTcM;
    double best = 1e300;
    for (int tn : cand) {
        for (int ks = 1; ks <= kTcMaxSplit && ks <= nk; ++ks) {
            const long long ctas = row_tiles * ((batch + tn - 1) / tn) * ks;
            const long long waves = (ctas + sm_count() - 1) / sm_count();
            const double alu = 900.0, mma = 8.4 * tn;
            const double cost = (double)waves * ((double)((nk + ks - 1) / ks) * (alu > mma ? alu : mma) + 3000.0);
            if (cost < best * 0.999) {
                best = cost;
                *tn_out = tn;
                *ks_out = ks;
            }
        }
    }
}

// W X as ks partial slices in scratch from the stream-ordered pool (the
// caller sums them and frees the scratch on the same stream).
// up != nullptr: x = up * silu(X) (row strides ldx, ldu), formed as x is read.
template <uint32_t FMT>
cudaError_t matmul_partials_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float **part_out,
                                int *ks_out, cudaStream_t s, const float *up = nullptr, int ldx = 0, int ldu = 0)
{
    const bool tc_ok = ((uintptr_t)X & 15u) == 0 &&
                       (up == nullptr || (((uintptr_t)up & 15u) == 0 && ldx % 4 == 0 && ldu % 4 == 0));
    const int nk = (L.cols + kTcK - 1) / kTcK;
    int tn = 0, ks = 1;
    if (g_matmul_path == 0 && batch >= kTcMinBatch && tc_ok) tc_split_plan(L.rows, batch, nk, &tn, &ks);
    cudaMemPool_t pool;
    cudaError_t e = scratch_pool(&pool);
    if (e != cudaSuccess) return e;
    const size_t n = (size_t)batch * (size_t)L.rows;
    void *part = nullptr;
    e = cudaMallocFromPoolAsync(&part, n * (size_t)ks * sizeof(float), pool, s);
    if (e != cudaSuccess) return e;
    float *P = (float *)part;
    const XSource src{X, up, up ? ldx : L.cols, ldu};
    void *xbuf = nullptr;
    if (tn == 0 && up) {  // the CUDA-core paths read a plain x: materialise up * silu(gate)
        e = cudaMallocFromPoolAsync(&xbuf, (size_t)batch * L.cols * sizeof(float), pool, s);
        if (e == cudaSuccess) {
            swiglu_rows_kernel<<<grid_for((uint64_t)batch * L.cols, kThreads), kThreads, 0, s>>>(
                X, ldx, up, ldu, L.cols, batch, (float *)xbuf);
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess) {
        switch (tn) {
        case 0: e = matmul_fmt<FMT>(L, w, xbuf ? (const float *)xbuf : X, batch, P, s); break;
        case 64: e = matmul_tc_go<FMT, 64>(L, w, src, batch, P, s, ks); break;
        case 128: e = matmul_tc_go<FMT, 128>(L, w, src, batch, P, s, ks); break;
        case 176: e = matmul_tc_go<FMT, 176>(L, w, src, batch, P, s, ks); break;
        default: e = matmul_tc_go<FMT, 256>(L, w, src, batch, P, s, ks); break;
        }
    }
    if (xbuf) cudaFreeAsync(xbuf, s);
    if (e != cudaSuccess) {
        cudaFreeAsync(part, s);
        return e;
    }
    *part_out = P;
    *ks_out = ks;
    return cudaSuccess;
}

// One CTA per row: h += the ks partial slices (in slice order), then
// out = (h / sqrt(mean(h^2) + eps)) * w (tensor_rms_norm_f32 of the updated
// residual stream).
__global__ void __launch_bounds__(kRowThreads)
rmsnorm_residual_kernel(float *__restrict__ h, const float *__restrict__ part, size_t slice, int ks,
                        const float *__restrict__ w, float eps, int cols, float *__restrict__ out)
{
    __shared__ float red[kRowThreads / 32];
    float *hr = h + (size_t)blockIdx.x * cols;
    const float *pr = part + (size_t)blockIdx.x * cols;
    float ss = 0.f;
    for (int i = threadIdx.x; i < cols; i += kRowThreads) {
        float acc = pr[i];
        for (int z = 1; z < ks; ++z) acc += pr[(size_t)z * slice + i];
        const float v = hr[i] + acc;
        hr[i] = v;
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int i = 0; i < kRowThreads / 32; ++i) ss += red[i];
    const float denom = sqrtf(ss / (float)cols + eps);
    float *orow = out + (size_t)blockIdx.x * cols;
    for (int i = threadIdx.x; i < cols; i += kRowThreads) orow[i] = (hr[i] / denom) * w[i];
}

template <uint32_t FMT>
cudaError_t matmul_residual_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float *H,
                                cudaStream_t s)
{
    float *P = nullptr;
    int ks = 1;
    cudaError_t e = matmul_partials_fmt<FMT>(L, w, X, batch, &P, &ks, s);
    if (e != cudaSuccess) return e;
    const size_t n = (size_t)batch * (size_t)L.rows;
    add_partials_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(H, P, n, ks);
    e = cudaGetLastError();
    const cudaError_t f = cudaFreeAsync(P, s);
    return e != cudaSuccess ? e : f;
}

}  // namespace

// ------------------------------------------------------------ exported

int block_elements(uint32_t type)
{
    switch (type) {
    case kQ5_0: case kQ8_0: return 32;
    case kQ4_K: case kQ6_K: return 256;
    default: return 0;
    }
}

int block_bytes(uint32_t type)
{
    switch (type) {
    case kQ5_0: return 22;
    case kQ8_0: return 34;
    case kQ4_K: return 144;
    case kQ6_K: return 210;
    default: return 0;
    }
}

bool make_layout(uint32_t type, int rows, int cols, Layout *out)
{
    const int be = block_elements(type);
    if (be == 0 || rows <= 0 || cols <= 0 || cols % be) return false;
    Layout L{};
    L.type = type;
    L.rows = rows;
    L.cols = cols;
    L.nb = cols / be;
    const uint32_t nb = (uint32_t)L.nb;
    switch (type) {
    case kQ8_0:
        L.C = L.nb;
        L.off_a = 32 * nb;
        L.row_stride = L.off_a + pad16(2 * nb);
        break;
    case kQ5_0:
        L.C = L.nb;
        L.off_a = 16 * nb;
        L.off_b = L.off_a + pad16(4 * nb);
        L.row_stride = L.off_b + pad16(2 * nb);
        break;
    case kQ4_K:
        L.C = 4 * L.nb;
        L.off_a = 128 * nb;
        L.row_stride = 144ull * nb;
        break;
    default:
        L.C = 4 * L.nb;
        L.off_a = 192 * nb;
        L.off_b = 208 * nb;
        L.row_stride = L.off_b + pad16(2 * nb);
        break;
    }
    *out = L;
    return true;
}

cudaError_t launch_repack(const Layout &L, const uint8_t *raw, uint8_t *dst, cudaStream_t s)
{
    cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)L.rows * L.row_stride, s);
    if (e != cudaSuccess) return e;
    const uint64_t n = (uint64_t)L.rows * L.C;
    repack_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(L, raw, dst);
    return cudaGetLastError();
}

cudaError_t launch_dequant_layout(const Layout &L, const uint8_t *w, float *out, cudaStream_t s)
{
    const unsigned g = grid_for((uint64_t)L.rows * L.nb, kThreads);
    switch (L.type) {
    case kQ8_0: dequant_layout_kernel<kQ8_0><<<g, kThreads, 0, s>>>(L, w, out); break;
    case kQ5_0: dequant_layout_kernel<kQ5_0><<<g, kThreads, 0, s>>>(L, w, out); break;
    case kQ4_K: dequant_layout_kernel<kQ4_K><<<g, kThreads, 0, s>>>(L, w, out); break;
    case kQ6_K: dequant_layout_kernel<kQ6_K><<<g, kThreads, 0, s>>>(L, w, out); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_raw(uint32_t type, const uint8_t *raw, uint64_t nblocks, float *out,
                               cudaStream_t s)
{
    const unsigned g = grid_for(nblocks * (uint64_t)block_elements(type), kThreads);
    switch (type) {
    case kQ8_0: dequant_raw_kernel<kQ8_0><<<g, kThreads, 0, s>>>(raw, nblocks, out); break;
    case kQ5_0: dequant_raw_kernel<kQ5_0><<<g, kThreads, 0, s>>>(raw, nblocks, out); break;
    case kQ4_K: dequant_raw_kernel<kQ4_K><<<g, kThreads, 0, s>>>(raw, nblocks, out); break;
    case kQ6_K: dequant_raw_kernel<kQ6_K><<<g, kThreads, 0, s>>>(raw, nblocks, out); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_embed(const Layout &L, const uint8_t *w, DecodeState *st, float *h, cudaStream_t s)
{
    const unsigned t = (unsigned)(L.nb < 256 ? L.nb : 256);
    switch (L.type) {
    case kQ8_0: embed_kernel<kQ8_0><<<1, t, 0, s>>>(L, w, st, h); break;
    case kQ5_0: embed_kernel<kQ5_0><<<1, t, 0, s>>>(L, w, st, h); break;
    case kQ4_K: embed_kernel<kQ4_K><<<1, t, 0, s>>>(L, w, st, h); break;
    case kQ6_K: embed_kernel<kQ6_K><<<1, t, 0, s>>>(L, w, st, h); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

size_t attention_workspace_floats(int heads, int kv_heads, int head_dim, int max_ctx)
{
    const size_t chunks = (size_t)(max_ctx + kAttnChunk - 1) / kAttnChunk;
    return (size_t)kv_heads * chunks * (size_t)(heads / kv_heads) * (size_t)(head_dim + 2);
}

cudaError_t launch_attention(const float *qkv, int heads, int kv_heads, int head_dim, float *kc, float *vc,
                             int max_ctx, float rope_base, DecodeState *st, float *part, unsigned int *counter,
                             float *att, cudaStream_t s)
{
    if (head_dim != 64 || kv_heads <= 0 || heads % kv_heads != 0 || heads / kv_heads > kAttnMaxGroup ||
        max_ctx <= 0)
        return cudaErrorInvalidValue;
    if (g_attn_path == 0 && heads / kv_heads <= kDaMaxGroup && attention_cluster_ok()) {
        cudaLaunchConfig_t cfg{};
        // two clusters per KV head (each half of the query heads) from 4 heads per group
        const int hsplit = heads / kv_heads >= 4 ? 2 : 1;
        cfg.gridDim = dim3((unsigned)(kv_heads * hsplit * kDaSplit));
        cfg.blockDim = dim3(kDaThreads);
        cfg.dynamicSmemBytes = kDaSmem;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = kDaSplit;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        return cudaLaunchKernelEx(&cfg, attention_cluster_kernel, qkv, heads, kv_heads, kc, vc, max_ctx, rope_base, st,
                                  att, hsplit);
    }
    const dim3 grid((unsigned)kv_heads, (unsigned)((max_ctx + kAttnChunk - 1) / kAttnChunk));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attention_kernel<64>, qkv, heads, kv_heads, kc, vc, max_ctx, rope_base, st, part,
                              counter, att);
}

void set_attention_path(int path) { g_attn_path = path; }

cudaError_t launch_advance(const unsigned long long *key, DecodeState *st, int *history, int max_steps,
                           cudaStream_t s, unsigned int *bar_count)
{
    advance_kernel<<<1, 1, 0, s>>>(key, st, history, max_steps, bar_count);
    return cudaGetLastError();
}

cudaError_t launch_embed_rows(const Layout &L, const uint8_t *w, const int *ids, int n, float *h,
                              unsigned int *err, cudaStream_t s)
{
    if (n <= 0) return cudaErrorInvalidValue;
    const int t = 128;
    switch (L.type) {
    case kQ8_0: embed_rows_kernel<kQ8_0><<<n, t, 0, s>>>(L, w, ids, h, err); break;
    case kQ5_0: embed_rows_kernel<kQ5_0><<<n, t, 0, s>>>(L, w, ids, h, err); break;
    case kQ4_K: embed_rows_kernel<kQ4_K><<<n, t, 0, s>>>(L, w, ids, h, err); break;
    case kQ6_K: embed_rows_kernel<kQ6_K><<<n, t, 0, s>>>(L, w, ids, h, err); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float eps, int cols, int rows, float *out,
                                cudaStream_t s)
{
    if (rows <= 0 || cols <= 0) return cudaErrorInvalidValue;
    rmsnorm_rows_kernel<<<rows, kRowThreads, 0, s>>>(x, w, eps, cols, out);
    return cudaGetLastError();
}

cudaError_t launch_rope_kv(float *q, int q_ld, const float *k, int k_ld, const float *v, int v_ld,
                           const float *bias_q, const float *bias_k, const float *bias_v, int heads, int kv_heads,
                           int head_dim, int pos0, int n, float rope_base, float *kc, float *vc, cudaStream_t s)
{
    if (head_dim != 64 || n <= 0) return cudaErrorInvalidValue;
    rope_kv_kernel<64><<<n, 128, 0, s>>>(q, q_ld, k, k_ld, v, v_ld, bias_q, bias_k, bias_v, heads, kv_heads, pos0,
                                         rope_base, kc, vc);
    return cudaGetLastError();
}

size_t prefill_attention_part_floats(int heads, int head_dim, int positions)
{
    return (size_t)positions * heads * kPfMaxSplits * (head_dim + 2);
}

cudaError_t launch_prefill_attention(const float *q, int q_ld, const float *kc, const float *vc, int heads,
                                     int kv_heads, int head_dim, int pos0, int n, float *att, float *part,
                                     unsigned int *counter, cudaStream_t s)
{
    const int G = heads / kv_heads;
    if (head_dim != 64 || n <= 0 || G < 1 || G > kPfRows || (q_ld & 1) || ((uintptr_t)q & 7u) ||
        ((uintptr_t)kc & 7u))
        return cudaErrorInvalidValue;
    if ((kv_heads * head_dim) % 4 || ((uintptr_t)kc & 15u) || ((uintptr_t)vc & 15u)) return cudaErrorInvalidValue;
    auto kernel = prefill_attention_kernel<64>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = allow_max_smem((const void *)kernel, dev);
    if (e != cudaSuccess) return e;
    const int qt = kPfRows / G;  // positions per CTA: qt * G rows <= kPfRows
    // at most 4 key tiles per CTA (a short causal critical path), at most
    // kPfMaxSplits splits per query block
    const int max_tiles = (pos0 + n - 1) / kPfKeys + 1;
    int tps = 4;
    if ((max_tiles + tps - 1) / tps > kPfMaxSplits) tps = (max_tiles + kPfMaxSplits - 1) / kPfMaxSplits;
    const int zs = (max_tiles + tps - 1) / tps;
    if (zs > 1 && part == nullptr) return cudaErrorInvalidValue;
    if (zs > 1 && counter == nullptr) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)kv_heads, (unsigned)((n + qt - 1) / qt), (unsigned)zs);
    kernel<<<grid, kPfWarps * 32, kPfSmem, s>>>(q, q_ld, kc, vc, heads, kv_heads, pos0, n, qt, tps, att, part,
                                                counter);
    return cudaGetLastError();
}

cudaError_t launch_gemv(const Layout &L, const uint8_t *w, const float *x, float *y,
                        const ArgmaxOut *am, cudaStream_t s)
{
    switch (L.type) {
    case kQ8_0: return gemv_fmt<kQ8_0>(L, w, x, y, am, s);
    case kQ5_0: return gemv_fmt<kQ5_0>(L, w, x, y, am, s);
    case kQ4_K: return gemv_fmt<kQ4_K>(L, w, x, y, am, s);
    case kQ6_K: return gemv_fmt<kQ6_K>(L, w, x, y, am, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv_fused(const Layout &L, const uint8_t *w, const float *x, float *y,
                              const ArgmaxOut *am, const Fuse &fu, cudaStream_t s)
{
    switch (L.type) {
    case kQ8_0: return gemv_fused_fmt<kQ8_0>(L, w, x, y, am, fu, s);
    case kQ5_0: return gemv_fused_fmt<kQ5_0>(L, w, x, y, am, fu, s);
    case kQ4_K: return gemv_fused_fmt<kQ4_K>(L, w, x, y, am, fu, s);
    case kQ6_K: return gemv_fused_fmt<kQ6_K>(L, w, x, y, am, fu, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv_pair(const Layout &La, const uint8_t *wa, float *ya, const Layout &Lb, const uint8_t *wb,
                             float *yb, const float *x, const Fuse &fu, cudaStream_t s)
{
    if (La.cols != Lb.cols || La.type == Lb.type || fu.add != nullptr || fu.pre == kPreSwiGlu)
        return cudaErrorInvalidValue;
    GemvPair pr = {};
    // ordered by format, so one instantiation serves both orders
    const bool swap = La.type > Lb.type;
    pr.L[0] = swap ? Lb : La;
    pr.L[1] = swap ? La : Lb;
    pr.w[0] = swap ? wb : wa;
    pr.w[1] = swap ? wa : wb;
    pr.y[0] = swap ? yb : ya;
    pr.y[1] = swap ? ya : yb;
    // Q5_0 and Q8_0 share the quantized x's slice layout: both matrices in
    // every CTA of one resident-row-range launch when their rows fit
    if (g_gemv_path == 5 && pr.L[0].type == kQ5_0 && pr.L[1].type == kQ8_0) {
        const LiteMat mats[2] = {{pr.L[0], pr.w[0], pr.y[0], nullptr, 0}, {pr.L[1], pr.w[1], pr.y[1], nullptr, 0}};
        LitePlan P;
        unsigned lgrid = 0;
        if (lite_plan(mats, 2, &P, &lgrid)) return gemv_lite_go<kQ5_0, kQ8_0>(P, lgrid, x, nullptr, fu, s);
    }
    // one CTA per SM, split between the matrices by their bytes
    const long long sms = sm_count();
    if (sms < 2) return cudaErrorNotSupported;
    const double b0 = (double)pr.L[0].rows * (double)pr.L[0].row_stride;
    const double b1 = (double)pr.L[1].rows * (double)pr.L[1].row_stride;
    long long c0 = (long long)(sms * b0 / (b0 + b1) + 0.5);
    if (c0 < 1) c0 = 1;
    if (c0 > sms - 1) c0 = sms - 1;
    if (c0 > pr.L[0].rows) c0 = pr.L[0].rows;
    long long c1 = sms - c0;
    if (c1 > pr.L[1].rows) c1 = pr.L[1].rows;
    pr.ctas0 = (int)c0;
    const int grid = (int)(c0 + c1);
    const uint32_t t0 = pr.L[0].type, t1 = pr.L[1].type;
#define QMV_PAIR(A, B) \
    if (t0 == A && t1 == B) return gemv_pair_fmt<A, B>(pr, grid, x, fu, s);
    QMV_PAIR(kQ5_0, kQ8_0)
    QMV_PAIR(kQ5_0, kQ4_K)
    QMV_PAIR(kQ5_0, kQ6_K)
    QMV_PAIR(kQ8_0, kQ4_K)
    QMV_PAIR(kQ8_0, kQ6_K)
    QMV_PAIR(kQ4_K, kQ6_K)
#undef QMV_PAIR
    return cudaErrorInvalidValue;
}

cudaError_t launch_matmul_partials(const Layout &L, const uint8_t *w, const float *X, int batch, float **part,
                                   int *ks, cudaStream_t s)
{
    if (batch <= 0) return cudaErrorInvalidValue;
    switch (L.type) {
    case kQ8_0: return matmul_partials_fmt<kQ8_0>(L, w, X, batch, part, ks, s);
    case kQ5_0: return matmul_partials_fmt<kQ5_0>(L, w, X, batch, part, ks, s);
    case kQ4_K: return matmul_partials_fmt<kQ4_K>(L, w, X, batch, part, ks, s);
    case kQ6_K: return matmul_partials_fmt<kQ6_K>(L, w, X, batch, part, ks, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_matmul_partials_swiglu(const Layout &L, const uint8_t *w, const float *gate, int g_ld,
                                          const float *up, int u_ld, int batch, float **part, int *ks, cudaStream_t s)
{
    if (batch <= 0 || gate == nullptr || up == nullptr) return cudaErrorInvalidValue;
    switch (L.type) {
    case kQ8_0: return matmul_partials_fmt<kQ8_0>(L, w, gate, batch, part, ks, s, up, g_ld, u_ld);
    case kQ5_0: return matmul_partials_fmt<kQ5_0>(L, w, gate, batch, part, ks, s, up, g_ld, u_ld);
    case kQ4_K: return matmul_partials_fmt<kQ4_K>(L, w, gate, batch, part, ks, s, up, g_ld, u_ld);
    case kQ6_K: return matmul_partials_fmt<kQ6_K>(L, w, gate, batch, part, ks, s, up, g_ld, u_ld);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rmsnorm_residual(float *h, const float *part, int ks, const float *w, float eps, int cols,
                                    int rows, float *out, cudaStream_t s)
{
    if (rows <= 0 || cols <= 0 || ks < 1) return cudaErrorInvalidValue;
    rmsnorm_residual_kernel<<<rows, kRowThreads, 0, s>>>(h, part, (size_t)rows * cols, ks, w, eps, cols, out);
    return cudaGetLastError();
}

cudaError_t launch_add_partials(float *h, const float *part, size_t n, int ks, cudaStream_t s)
{
    add_partials_kernel<<<grid_for(n, kThreads), kThreads, 0, s>>>(h, part, n, ks);
    return cudaGetLastError();
}

cudaError_t launch_matmul_residual(const Layout &L, const uint8_t *w, const float *X, int batch, float *H,
                                   cudaStream_t s)
{
    if (batch <= 0) return cudaErrorInvalidValue;
    switch (L.type) {
    case kQ8_0: return matmul_residual_fmt<kQ8_0>(L, w, X, batch, H, s);
    case kQ5_0: return matmul_residual_fmt<kQ5_0>(L, w, X, batch, H, s);
    case kQ4_K: return matmul_residual_fmt<kQ4_K>(L, w, X, batch, H, s);
    case kQ6_K: return matmul_residual_fmt<kQ6_K>(L, w, X, batch, H, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_matmul(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                          cudaStream_t s)
{
    switch (L.type) {
    case kQ8_0: return matmul_fmt<kQ8_0>(L, w, X, batch, Y, s);
    case kQ5_0: return matmul_fmt<kQ5_0>(L, w, X, batch, Y, s);
    case kQ4_K: return matmul_fmt<kQ4_K>(L, w, X, batch, Y, s);
    case kQ6_K: return matmul_fmt<kQ6_K>(L, w, X, batch, Y, s);
    default: return cudaErrorInvalidValue;
    }
}

void set_gemv_path(int path) { g_gemv_path = path; }
void set_call_status(unsigned int *word) { t_call_status = word; }
void set_matmul_path(int path) { g_matmul_path = path; }

size_t exchange_parity_bytes(int world, int slot_rows)
{
    const size_t logits = ((size_t)world * slot_rows * 4 + 255) & ~(size_t)255;
    return logits + (size_t)world * kMaxExCtas * (8 + 4);
}

cudaError_t launch_gemv_exchange(const Layout &L, const uint8_t *w, const float *x, float *y,
                                 const ArgmaxOut &am, const Exchange &ex, cudaStream_t s)
{
    switch (L.type) {
    case kQ8_0: return gemv_exchange_fmt<kQ8_0>(L, w, x, y, am, ex, s);
    case kQ5_0: return gemv_exchange_fmt<kQ5_0>(L, w, x, y, am, ex, s);
    case kQ4_K: return gemv_exchange_fmt<kQ4_K>(L, w, x, y, am, ex, s);
    case kQ6_K: return gemv_exchange_fmt<kQ6_K>(L, w, x, y, am, ex, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t read_status(unsigned int *out, bool clear)
{
    unsigned int peer = 0u;
    cudaError_t e = cudaMemcpyFromSymbol(out, g_status, sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&peer, g_peer_status, sizeof(unsigned int));
    if (e == cudaSuccess && peer) *out |= 8u;
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0u;
        e = cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned int));
        if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(unsigned int));
    }
    return e;
}

cudaError_t launch_argmax(const float *logits, int n, const ArgmaxOut &am, cudaStream_t s)
{
    unsigned g = grid_for((uint64_t)n, kThreads * 4);
    if (g > (unsigned)kMaxArgmaxCtas) g = kMaxArgmaxCtas;
    argmax_kernel<<<g, kThreads, 0, s>>>(logits, n, am);
    return cudaGetLastError();
}

// ------------------------------------------------- persistent decode step

size_t decode_layers_smem(int dim, int hid, uint32_t slot_bytes)
{
    return (size_t)ps_x_bytes(dim, hid) + sizeof(float) * (size_t)kPsParts + 2u * (size_t)slot_bytes;
}

// Weight slot size: two slots in what the x area, the partial sums and the
// static tiles leave of the opt-in shared memory, at most 64 KiB each, a
// multiple of 128 bytes.
uint32_t decode_layers_slot_bytes(int dim, int hid)
{
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return 0;
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, decode_layers_kernel) != cudaSuccess) return 0;
    const long long left =
        (long long)optin - (long long)attr.sharedSizeBytes - (long long)ps_x_bytes(dim, hid) - 4ll * kPsParts;
    long long slot = left / 2;
    if (slot > 64 * 1024) slot = 64 * 1024;
    return slot > 0 ? (uint32_t)(slot / 128 * 128) : 0u;
}

cudaError_t launch_decode_layers(const PStep &P, cudaStream_t s)
{
    if (P.heads <= 0 || P.kv_heads <= 0 || P.heads % P.kv_heads != 0 || P.heads / P.kv_heads > kAttnMaxGroup ||
        P.max_ctx <= 0 || P.dim != P.heads * 64)
        return cudaErrorInvalidValue;
    const size_t smem = decode_layers_smem(P.dim, P.hid, P.slot_bytes);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = allow_max_smem((const void *)decode_layers_kernel, dev);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_layers_kernel, kPsThreads, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sm_count());  // one CTA per SM, all resident (cooperative)
    cfg.blockDim = dim3(kPsThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_layers_kernel, P);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------- argmax without allocation
//
// For callers that cannot call cudaMalloc (a host that owns every device
// allocation through its own pool and hands a plugin only input and output
// buffers): the argmax scratch -- the arrival counter and the running maximum
// key in its first 16 bytes, then room for one key per CTA (the layout of the
// caller workspace of qmv_argmax) -- lives in this file-scope device array
// instead of a caller workspace.  One CTA covers kNoAllocLogitsPerCta logits,
// and a call is bounded at kNoAllocMaxCtas CTAs (kNoAllocMaxLogits logits).  Every GPU that loads the library holds the array
// until the process exits.  All calls on a device share it and it keeps the
// last call's contents: each call clears the counter first, and calls that
// overlap on the GPU (concurrent streams) race on it.

namespace {
constexpr int kNoAllocMaxCtas = 2048;
constexpr int kNoAllocLogitsPerCta = 4096;
static __device__ __align__(256) unsigned char g_noalloc_scratch[16 + 8 * kNoAllocMaxCtas];

std::mutex g_noalloc_mutex;
void *g_noalloc_ptr[256];  // device address of g_noalloc_scratch per device
}  // namespace

int noalloc_max_logits() { return kNoAllocMaxCtas * kNoAllocLogitsPerCta; }

// Device address of the scratch array on the current device.  Host code only
// knows a host-side stand-in for the symbol, so the address is looked up once
// per device (with that device current) and cached.  The address belongs to
// the CUDA runtime's primary context of that device, the one every runtime
// call of this library uses; it does not survive a cudaDeviceReset, and a
// host driving the library from a context of its own must not use this entry
// point.
static cudaError_t noalloc_scratch(void **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 256) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

cudaError_t launch_argmax_noalloc(const float *logits, int n, int index_base, unsigned long long *key,
                                  cudaStream_t s)
{
    if (n <= 0 || n > noalloc_max_logits()) return cudaErrorInvalidValue;
    void *scratch = nullptr;
    cudaError_t e = noalloc_scratch(&scratch);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(scratch, 0, 16, s);  // arrival counter and running maximum start at zero
    if (e != cudaSuccess) return e;
    const unsigned g = (unsigned)((n + kNoAllocLogitsPerCta - 1) / kNoAllocLogitsPerCta);
    argmax_kernel<<<g, kThreads, 0, s>>>(logits, n, ArgmaxOut{key, scratch, index_base});
    return cudaGetLastError();
}

}  // namespace qmv
