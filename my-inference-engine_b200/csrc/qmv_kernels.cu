// sm_100a kernels for the GGUF quantized matrix-vector path.
//
//  * repack      raw GGUF blocks -> 16-byte-aligned resident rows (once).
//  * dequant     bit-exact block decoding (same float bits as the reference's
//                *_dequantize_block, src/quantization.cpp:54-67, 161-184,
//                380-409, 588-615).
//  * gemv        y = W x, in-register dequantisation with dp4a integer dots.
//  * matmul      Y = W X for a batch of positions, each weight block loaded
//                once and applied to every position
//                (src/quantized_matvec.cpp:164-224).
//  * argmax      greedy selection fused into the gemv epilogue, or alone
//                (src/sampler.cpp:14-36).
//
// Integer inner loop.  Each 32-element block j of x is quantized on the fly
// into 16-bit integers xq = rint(x / s_j) held as two int8 planes
// (hi = (xq + 128) >> 8, lo = xq - 256 hi), where s_j is the power of two
// that puts max|xq| in (16320, 32639].  A block dot is then
// s_j * (256 * dp4a(w, hi) + dp4a(w, lo)) with exact 32-bit integer sums; the
// quantisation error of x is at most 2^-15 of the block maximum (none at all
// for dyadic inputs), far inside the parity bound
// |y - y_ref| <= 1e-4 * sum|w x|.  Blocks whose maximum is below 2^-100 share
// the scale 2^-114, so magnitudes under 2^-115 quantize to zero.
// Offsets of Q5_0 (-16) and Q6_K (-32) are folded in with per-16-element sums
// of xq; the Q4_K minimum uses the same sums.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

__device__ __forceinline__ uint2 ld_stream8(const uint8_t *p)
{
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p)
{
    return __ldg(reinterpret_cast<const unsigned int *>(p));
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p)
{
    return __ldg(reinterpret_cast<const unsigned short *>(p));
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

// Publish this CTA's key; the last CTA to arrive folds all of them into
// *out and re-arms the counter.  No CTA waits on another.
__device__ void finish_argmax(unsigned long long cta_key, const ArgmaxOut &am,
                              unsigned long long *scratch)
{
    unsigned int *counter = reinterpret_cast<unsigned int *>(am.workspace);
    unsigned long long *keys =
        reinterpret_cast<unsigned long long *>(reinterpret_cast<uint8_t *>(am.workspace) + 16);
    __shared__ int is_last;
    if (threadIdx.x == 0) {
        keys[blockIdx.x] = cta_key;
        __threadfence();
        unsigned int prev = atomicAdd(counter, 1u);
        is_last = (prev == gridDim.x - 1u);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    unsigned long long k = 0ull;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x)
        k = max_ull(k, __ldcg(keys + i));
    k = block_max_key(k, scratch);
    if (threadIdx.x == 0) {
        *am.key = k;
        *counter = 0u;
    }
}

// ------------------------------------------------------- x quantisation

struct XS {
    const int8_t *xh;   // [cols]
    const int8_t *xl;   // [cols]
    const float *xs;    // [cols/32] block scale (NaN if the block is non-finite)
    const int *xsum;    // [cols/16] sum of xq over 16 elements
};

// Bytes of one quantized position, rounded up to 16 so that consecutive
// positions keep the 16-byte alignment of their 128-bit shared loads.
__host__ __device__ constexpr size_t xs_bytes(int cols)
{
    return (2 * (size_t)cols + (size_t)cols / 8 + (size_t)cols / 4 + 15) & ~(size_t)15;
}

__device__ __forceinline__ XS xs_view(uint8_t *base, int cols)
{
    XS s;
    s.xh = reinterpret_cast<const int8_t *>(base);
    s.xl = reinterpret_cast<const int8_t *>(base + cols);
    s.xs = reinterpret_cast<const float *>(base + 2 * cols);
    s.xsum = reinterpret_cast<const int *>(base + 2 * cols + cols / 8);
    return s;
}

// Quantize x[0..cols) into shared memory (all threads of the CTA take part;
// 8 consecutive lanes own one 32-element block).
__device__ void quantize_x(const float *__restrict__ x, int cols, uint8_t *base)
{
    uint32_t *xh = reinterpret_cast<uint32_t *>(base);
    uint32_t *xl = reinterpret_cast<uint32_t *>(base + cols);
    float *xs = reinterpret_cast<float *>(base + 2 * cols);
    int *xsum = reinterpret_cast<int *>(base + 2 * cols + cols / 8);
    const int n4 = cols >> 2;
    const int lane = threadIdx.x & 31;
    constexpr int U = 8;
    for (int it0 = 0; it0 * kThreads < n4; it0 += U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int f = (it0 + u) * kThreads + threadIdx.x;
            v[u] = f < n4 ? __ldg(reinterpret_cast<const float4 *>(x) + f)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if ((it0 + u) * kThreads >= n4) break;  // uniform across the CTA
            const int f = (it0 + u) * kThreads + threadIdx.x;
            uint32_t a = max(max(__float_as_uint(fabsf(v[u].x)), __float_as_uint(fabsf(v[u].y))),
                             max(__float_as_uint(fabsf(v[u].z)), __float_as_uint(fabsf(v[u].w))));
            a = max(a, __shfl_xor_sync(kFull, a, 1));
            a = max(a, __shfl_xor_sync(kFull, a, 2));
            a = max(a, __shfl_xor_sync(kFull, a, 4));
            // Power-of-two scale s = 2^e with |x| / s <= 32639: x * 2^-e is
            // exact, so dyadic inputs (small integers, k/2^n) stay exact.
            const bool bad = a >= 0x7f800000u;
            const int ea = max((int)(a >> 23), 27);  // blocks below 2^-100 share 2^-114
            int e = ea - 127 - 14;
            float inv = __uint_as_float((uint32_t)(127 - e) << 23);
            if (__uint_as_float(a) * inv >= 32639.5f) {
                e += 1;
                inv *= 0.5f;
            }
            if (bad) inv = 0.f;
            int q0 = __float2int_rn(v[u].x * inv), q1 = __float2int_rn(v[u].y * inv);
            int q2 = __float2int_rn(v[u].z * inv), q3 = __float2int_rn(v[u].w * inv);
            int h0 = (q0 + 128) >> 8, h1 = (q1 + 128) >> 8, h2 = (q2 + 128) >> 8, h3 = (q3 + 128) >> 8;
            int l0 = q0 - (h0 << 8), l1 = q1 - (h1 << 8), l2 = q2 - (h2 << 8), l3 = q3 - (h3 << 8);
            uint32_t hh = (uint32_t)(h0 & 0xff) | ((uint32_t)(h1 & 0xff) << 8) |
                          ((uint32_t)(h2 & 0xff) << 16) | ((uint32_t)(h3 & 0xff) << 24);
            uint32_t ll = (uint32_t)(l0 & 0xff) | ((uint32_t)(l1 & 0xff) << 8) |
                          ((uint32_t)(l2 & 0xff) << 16) | ((uint32_t)(l3 & 0xff) << 24);
            int s4 = q0 + q1 + q2 + q3;
            s4 += __shfl_xor_sync(kFull, s4, 1);
            s4 += __shfl_xor_sync(kFull, s4, 2);
            if (f < n4) {
                xh[f] = hh;
                xl[f] = ll;
                if ((lane & 3) == 0) xsum[f >> 2] = s4;
                if ((lane & 7) == 0)
                    xs[f >> 3] = bad ? __uint_as_float(0x7fc00000u) : __uint_as_float((uint32_t)(127 + e) << 23);
            }
        }
    }
}

// ------------------------------------------------- per-format chunk code
//
// A "chunk" is the unit one thread handles per row: a whole 32-weight block
// for Q8_0/Q5_0, 64 weights (two sub-blocks / four 16-element scale groups)
// for Q4_K/Q6_K.  W<FMT> holds one row's chunk in registers; load() issues the
// global loads, dot() consumes x from shared memory.

template <uint32_t FMT> struct Chunk;

template <> struct Chunk<kQ8_0> {
    uint4 a, b;
    uint32_t d;
    static __host__ __device__ int per_row(int cols) { return cols / 32; }
    __device__ void load(const uint8_t *row, const Layout &L, int c)
    {
        a = ld_stream(row + 32 * c);
        b = ld_stream(row + 32 * c + 16);
        d = ld_u16(row + L.off_d + 2 * c);
    }
    __device__ float dot(const XS &s, int c) const
    {
        const uint4 *h = reinterpret_cast<const uint4 *>(s.xh + 32 * c);
        const uint4 *l = reinterpret_cast<const uint4 *>(s.xl + 32 * c);
        uint4 h0 = h[0], h1 = h[1], l0 = l[0], l1 = l[1];
        int ah = dp4a(a.x, h0.x, 0);
        ah = dp4a(a.y, h0.y, ah); ah = dp4a(a.z, h0.z, ah); ah = dp4a(a.w, h0.w, ah);
        ah = dp4a(b.x, h1.x, ah); ah = dp4a(b.y, h1.y, ah); ah = dp4a(b.z, h1.z, ah); ah = dp4a(b.w, h1.w, ah);
        int al = dp4a(a.x, l0.x, 0);
        al = dp4a(a.y, l0.y, al); al = dp4a(a.z, l0.z, al); al = dp4a(a.w, l0.w, al);
        al = dp4a(b.x, l1.x, al); al = dp4a(b.y, l1.y, al); al = dp4a(b.z, l1.z, al); al = dp4a(b.w, l1.w, al);
        return (f16_fast(d) * s.xs[c]) * (float)(ah * 256 + al);
    }
};

// Spread bits 0..3 of v to bit 4 of bytes 0..3.
__device__ __forceinline__ uint32_t spread4(uint32_t v)
{
    return ((v & 0xfu) * 0x02040810u) & 0x10101010u;
}

template <> struct Chunk<kQ5_0> {
    uint4 q;
    uint32_t qh, d;
    static __host__ __device__ int per_row(int cols) { return cols / 32; }
    __device__ void load(const uint8_t *row, const Layout &L, int c)
    {
        q = ld_stream(row + 16 * c);
        qh = ld_u32(row + L.off_qh + 4 * c);
        d = ld_u16(row + L.off_d + 2 * c);
    }
    __device__ float dot(const XS &s, int c) const
    {
        const uint4 *h = reinterpret_cast<const uint4 *>(s.xh + 32 * c);
        const uint4 *l = reinterpret_cast<const uint4 *>(s.xl + 32 * c);
        uint4 h0 = h[0], h1 = h[1], l0 = l[0], l1 = l[1];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        const uint32_t xh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t xl[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        int ah = 0, al = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // weights 4k..4k+3: low nibbles; weights 16+4k..: high nibbles
            uint32_t lo = (w[k] & 0x0f0f0f0fu) | spread4(qh >> (4 * k));
            uint32_t hi = ((w[k] >> 4) & 0x0f0f0f0fu) | spread4(qh >> (16 + 4 * k));
            ah = dp4a(lo, xh[k], ah);
            al = dp4a(lo, xl[k], al);
            ah = dp4a(hi, xh[4 + k], ah);
            al = dp4a(hi, xl[4 + k], al);
        }
        const int sx = s.xsum[2 * c] + s.xsum[2 * c + 1];
        return (f16_fast(d) * s.xs[c]) * (float)(ah * 256 + al - 16 * sx);
    }
};

template <> struct Chunk<kQ4_K> {
    uint4 hdr, a, b;
    static __host__ __device__ int per_row(int cols) { return cols / 64; }
    __device__ void load(const uint8_t *row, const Layout &, int c)
    {
        const uint8_t *blk = row + 144 * (c >> 2);
        hdr = ld_stream(blk);
        a = ld_stream(blk + 16 + 32 * (c & 3));
        b = ld_stream(blk + 32 + 32 * (c & 3));
    }
    __device__ float dot(const XS &s, int c) const
    {
        const int g = c & 3;
        const uint4 *h = reinterpret_cast<const uint4 *>(s.xh + 64 * c);
        const uint4 *l = reinterpret_cast<const uint4 *>(s.xl + 64 * c);
        const uint32_t q[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        int ah0 = 0, al0 = 0, ah1 = 0, al1 = 0;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            uint4 xh0 = h[k], xl0 = l[k], xh1 = h[2 + k], xl1 = l[2 + k];
            const uint32_t xa[4] = {xh0.x, xh0.y, xh0.z, xh0.w};
            const uint32_t xb[4] = {xl0.x, xl0.y, xl0.z, xl0.w};
            const uint32_t xc[4] = {xh1.x, xh1.y, xh1.z, xh1.w};
            const uint32_t xd[4] = {xl1.x, xl1.y, xl1.z, xl1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t lo = q[4 * k + j] & 0x0f0f0f0fu;         // sub-block 2g
                uint32_t hi = (q[4 * k + j] >> 4) & 0x0f0f0f0fu;  // sub-block 2g+1
                ah0 = dp4a(lo, xa[j], ah0);
                al0 = dp4a(lo, xb[j], al0);
                ah1 = dp4a(hi, xc[j], ah1);
                al1 = dp4a(hi, xd[j], al1);
            }
        }
        // 6-bit scale / min of sub-blocks 2g and 2g+1 (src/quantization.cpp:351-378)
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
        uint32_t sc0, m0, sc1, m1;
        if (g < 2) {
            const int t0 = 16 * g, t1 = 16 * g + 8;
            sc0 = (s0 >> t0) & 63u; m0 = (s1 >> t0) & 63u;
            sc1 = (s0 >> t1) & 63u; m1 = (s1 >> t1) & 63u;
        } else {
            const int t0 = 16 * (g - 2), t1 = t0 + 8;
            sc0 = ((s2 >> t0) & 15u) | (((s0 >> t0) >> 6 & 3u) << 4);
            m0 = ((s2 >> t0) >> 4 & 15u) | (((s1 >> t0) >> 6 & 3u) << 4);
            sc1 = ((s2 >> t1) & 15u) | (((s0 >> t1) >> 6 & 3u) << 4);
            m1 = ((s2 >> t1) >> 4 & 15u) | (((s1 >> t1) >> 6 & 3u) << 4);
        }
        const float d = f16_fast(hdr.x), dmin = f16_fast(hdr.x >> 16);
        const int j0 = 2 * c;  // 32-element x block of sub-block 2g
        const int S0 = s.xsum[2 * j0] + s.xsum[2 * j0 + 1];
        const int S1 = s.xsum[2 * j0 + 2] + s.xsum[2 * j0 + 3];
        const float v0 = (d * (float)sc0) * (float)(ah0 * 256 + al0) - (dmin * (float)m0) * (float)S0;
        const float v1 = (d * (float)sc1) * (float)(ah1 * 256 + al1) - (dmin * (float)m1) * (float)S1;
        return s.xs[j0] * v0 + s.xs[j0 + 1] * v1;
    }
};

template <> struct Chunk<kQ6_K> {
    uint4 l0, l1, qh;
    uint2 sc;
    uint32_t d;
    static __host__ __device__ int per_row(int cols) { return cols / 64; }
    __device__ void load(const uint8_t *row, const Layout &L, int c)
    {
        const int sb = c >> 2, g = (c >> 1) & 1, h = c & 1;
        const uint8_t *blk = row + 208 * sb;
        l0 = ld_stream(blk + 64 * g + 16 * h);
        l1 = ld_stream(blk + 64 * g + 32 + 16 * h);
        qh = ld_stream(blk + 128 + 32 * g + 16 * h);
        sc = ld_stream8(blk + 192 + 8 * g);
        d = ld_u16(row + L.off_d + 2 * sb);
    }
    __device__ float dot(const XS &s, int c) const
    {
        // positions of region r: 128*(c>>1) + 16*(c&1) + 32*r
        const int base = 128 * (c >> 1) + 16 * (c & 1);
        const int h = c & 1;
        const uint32_t a[4] = {l0.x, l0.y, l0.z, l0.w};
        const uint32_t b[4] = {l1.x, l1.y, l1.z, l1.w};
        const uint32_t u[4] = {qh.x, qh.y, qh.z, qh.w};
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint4 xh4 = *reinterpret_cast<const uint4 *>(s.xh + base + 32 * r);
            const uint4 xl4 = *reinterpret_cast<const uint4 *>(s.xl + base + 32 * r);
            const uint32_t xa[4] = {xh4.x, xh4.y, xh4.z, xh4.w};
            const uint32_t xb[4] = {xl4.x, xl4.y, xl4.z, xl4.w};
            int ah = 0, al = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t lowbits, highbits;
                if (r == 0) { lowbits = a[k] & 0x0f0f0f0fu; highbits = (u[k] << 4) & 0x30303030u; }
                else if (r == 1) { lowbits = b[k] & 0x0f0f0f0fu; highbits = (u[k] << 2) & 0x30303030u; }
                else if (r == 2) { lowbits = (a[k] >> 4) & 0x0f0f0f0fu; highbits = u[k] & 0x30303030u; }
                else { lowbits = (b[k] >> 4) & 0x0f0f0f0fu; highbits = (u[k] >> 2) & 0x30303030u; }
                const uint32_t w = lowbits | highbits;  // 6-bit values 0..63
                ah = dp4a(w, xa[k], ah);
                al = dp4a(w, xb[k], al);
            }
            const int S = s.xsum[(base >> 4) + 2 * r];
            // int8 scale sc[8g + 2r + h]: byte (2r + h) of the loaded 8 bytes
            const uint32_t sw = (r < 2) ? sc.x : sc.y;
            const int scale = (int)(int8_t)((sw >> (8 * ((2 * r + h) & 3))) & 0xffu);
            acc += ((float)scale * s.xs[(base >> 5) + r]) * (float)(ah * 256 + al - 32 * S);
        }
        return f16_fast(d) * acc;
    }
};

// ---------------------------------------------------------------- GEMV
//
// Persistent CTAs, each owning a contiguous range of rows [r0, r1).  Inside
// a CTA, groups of TPT threads each take R consecutive rows per pass; the
// TPT threads of a group stride over the row's chunks, so the x chunk in
// registers serves R rows.  Reductions are shuffle trees in a fixed order,
// so results are deterministic.

template <int R> struct RowAcc { float v[R]; };

template <uint32_t FMT, int TPT, int R>
__global__ void __launch_bounds__(kThreads)
gemv_kernel(Layout L, const uint8_t *__restrict__ w, const float *__restrict__ x,
            float *__restrict__ y, ArgmaxOut am, int want_argmax)
{
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float red[kThreads / 32][R];
    __shared__ unsigned long long kscratch[kThreads / 32];

    const int cols = L.cols;
    quantize_x(x, cols, smem);
    __syncthreads();
    const XS s = xs_view(smem, cols);

    const int r0 = (int)((long long)L.rows * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)L.rows * (blockIdx.x + 1) / gridDim.x);
    constexpr int NG = kThreads / TPT;
    const int group = threadIdx.x / TPT, gl = threadIdx.x % TPT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = Chunk<FMT>::per_row(cols);
    const int passes = (r1 - r0 + NG * R - 1) / (NG * R);
    unsigned long long best = 0ull;

    for (int ps = 0; ps < passes; ++ps) {
        const int row0 = r0 + (ps * NG + group) * R;
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.f;
        for (int c = gl; c < C; c += TPT) {
            Chunk<FMT> ch[R];
#pragma unroll
            for (int i = 0; i < R; ++i)
                if (row0 + i < r1) ch[i].load(w + (uint64_t)(row0 + i) * L.row_stride, L, c);
#pragma unroll
            for (int i = 0; i < R; ++i)
                if (row0 + i < r1) acc[i] += ch[i].dot(s, c);
        }
        constexpr int WL = TPT < 32 ? TPT : 32;
#pragma unroll
        for (int i = 0; i < R; ++i) {
#pragma unroll
            for (int o = WL / 2; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(kFull, acc[i], o);
        }
        float out = 0.f;
        if constexpr (TPT > 32) {
            if (lane == 0) {
#pragma unroll
                for (int i = 0; i < R; ++i) red[warp][i] = acc[i];
            }
            __syncthreads();
            if (gl < R) {
                constexpr int WPG = TPT / 32;
                for (int k = 0; k < WPG; ++k) out += red[group * WPG + k][gl];
            }
            __syncthreads();
        } else {
#pragma unroll
            for (int i = 0; i < R; ++i)
                if (gl == i) out = acc[i];
        }
        if (gl < R) {
            const int row = row0 + gl;
            if (row < r1) {
                y[row] = out;
                if (want_argmax) best = max_ull(best, make_key(out, am.index_base + row));
            }
        }
    }
    if (want_argmax) {
        best = block_max_key(best, kscratch);
        finish_argmax(best, am, kscratch);
    }
}

// ------------------------------------------------------------- matmul
//
// Batched form: NP <= 8 positions share every weight chunk load.  x of all
// positions is quantized into shared memory first.

template <uint32_t FMT, int TPT, int NP>
__global__ void __launch_bounds__(kThreads)
matmul_kernel(Layout L, const uint8_t *__restrict__ w, const float *__restrict__ X, int np,
              float *__restrict__ Y)
{
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float red[kThreads / 32][NP];
    const int cols = L.cols;
    const size_t xb = xs_bytes(cols);
    for (int p = 0; p < np; ++p) quantize_x(X + (size_t)p * cols, cols, smem + p * xb);
    __syncthreads();

    const int r0 = (int)((long long)L.rows * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)L.rows * (blockIdx.x + 1) / gridDim.x);
    constexpr int NG = kThreads / TPT;
    const int group = threadIdx.x / TPT, gl = threadIdx.x % TPT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = Chunk<FMT>::per_row(cols);
    const int passes = (r1 - r0 + NG - 1) / NG;

    for (int ps = 0; ps < passes; ++ps) {
        const int row = r0 + ps * NG + group;
        float acc[NP];
#pragma unroll
        for (int p = 0; p < NP; ++p) acc[p] = 0.f;
        if (row < r1) {
            const uint8_t *rp = w + (uint64_t)row * L.row_stride;
            for (int c = gl; c < C; c += TPT) {
                Chunk<FMT> ch;
                ch.load(rp, L, c);
#pragma unroll
                for (int p = 0; p < NP; ++p)
                    if (p < np) acc[p] += ch.dot(xs_view(smem + p * xb, cols), c);
            }
        }
        constexpr int WL = TPT < 32 ? TPT : 32;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
#pragma unroll
            for (int o = WL / 2; o > 0; o >>= 1) acc[p] += __shfl_xor_sync(kFull, acc[p], o);
        }
        float out = 0.f;
        if constexpr (TPT > 32) {
            if (lane == 0) {
#pragma unroll
                for (int p = 0; p < NP; ++p) red[warp][p] = acc[p];
            }
            __syncthreads();
            if (gl < np) {
                constexpr int WPG = TPT / 32;
                for (int k = 0; k < WPG; ++k) out += red[group * WPG + k][gl];
            }
            __syncthreads();
        } else {
#pragma unroll
            for (int p = 0; p < NP; ++p)
                if (gl == p) out = acc[p];
        }
        if (gl < np && row < r1) Y[(size_t)gl * L.rows + row] = out;
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

__global__ void repack_kernel(Layout L, const uint8_t *__restrict__ raw, uint8_t *__restrict__ dst)
{
    const uint64_t nblocks = (uint64_t)L.rows * L.nb;
    const int bb = (L.type == kQ8_0) ? 34 : (L.type == kQ5_0) ? 22 : (L.type == kQ4_K) ? 144 : 210;
    for (uint64_t b = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; b < nblocks;
         b += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = b / L.nb;
        const int j = (int)(b % L.nb);
        const uint8_t *src = raw + b * bb;
        uint8_t *r = dst + row * L.row_stride;
        switch (L.type) {
        case kQ8_0:
            r[L.off_d + 2 * j] = src[0];
            r[L.off_d + 2 * j + 1] = src[1];
            for (int k = 0; k < 32; ++k) r[32 * j + k] = src[2 + k];
            break;
        case kQ5_0:
            r[L.off_d + 2 * j] = src[0];
            r[L.off_d + 2 * j + 1] = src[1];
            for (int k = 0; k < 4; ++k) r[L.off_qh + 4 * j + k] = src[2 + k];
            for (int k = 0; k < 16; ++k) r[16 * j + k] = src[6 + k];
            break;
        case kQ4_K:
            for (int k = 0; k < 144; ++k) r[144 * j + k] = src[k];
            break;
        default:
            for (int k = 0; k < 208; ++k) r[208 * j + k] = src[k];
            r[L.off_d + 2 * j] = src[208];
            r[L.off_d + 2 * j + 1] = src[209];
            break;
        }
    }
}

// Pointers to the fields of one block, wherever they live.
struct BlockRef {
    uint32_t d16;        // Q8_0/Q5_0/Q6_K scale bits
    const uint8_t *p;    // Q8_0 qs / Q5_0 qs / Q4_K whole block / Q6_K payload
    const uint8_t *qh;   // Q5_0 high bits
};

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

// Value i of a block, with the reference's rounding sequence (no FMA).
template <uint32_t FMT>
__device__ __forceinline__ float dequant_value(const BlockRef &b, int i)
{
    if constexpr (FMT == kQ8_0) {
        return mul_ref(f16_exact(b.d16), (float)(int8_t)b.p[i]);
    } else if constexpr (FMT == kQ5_0) {
        const int nib = i < 16 ? (b.p[i] & 0x0f) : (b.p[i - 16] >> 4);
        const int hi = (b.qh[i >> 3] >> (i & 7)) & 1;
        return mul_ref(f16_exact(b.d16), (float)((nib | (hi << 4)) - 16));
    } else if constexpr (FMT == kQ4_K) {
        const uint8_t *sm = b.p + 4;
        const int j = i >> 5, o = i & 31;
        int sc, mn;
        if (j < 4) {
            sc = sm[j] & 63;
            mn = sm[j + 4] & 63;
        } else {
            sc = (sm[j + 4] & 0x0f) | ((sm[j - 4] >> 6) << 4);
            mn = (sm[j + 4] >> 4) | ((sm[j] >> 6) << 4);
        }
        const float d = f16_exact((uint32_t)b.p[0] | ((uint32_t)b.p[1] << 8));
        const float dmin = f16_exact((uint32_t)b.p[2] | ((uint32_t)b.p[3] << 8));
        const float scale = mul_ref(d, (float)sc);
        const float minimum = mul_ref(dmin, (float)mn);
        const int nib = (b.p[16 + 32 * (j >> 1) + o] >> (4 * (j & 1))) & 0x0f;
        return sub_ref(mul_ref(scale, (float)nib), minimum);
    } else {
        const int g = i >> 7, loc = i & 127, r = loc >> 5, o = loc & 31;
        const int lo = (b.p[64 * g + 32 * (r & 1) + o] >> (4 * (r >> 1))) & 0x0f;
        const int hi = (b.p[128 + 32 * g + o] >> (2 * r)) & 0x03;
        const int q = (lo | (hi << 4)) - 32;
        const int sc = (int8_t)b.p[192 + 8 * g + 2 * r + (o >> 4)];
        return mul_ref(mul_ref(f16_exact(b.d16), (float)sc), (float)q);
    }
}

template <uint32_t FMT>
__device__ __forceinline__ BlockRef ref_layout(const Layout &L, const uint8_t *w, uint64_t row, int j)
{
    const uint8_t *r = w + row * L.row_stride;
    BlockRef b;
    b.qh = nullptr;
    b.d16 = 0;
    if constexpr (FMT == kQ8_0) {
        b.p = r + 32 * j;
        b.d16 = (uint32_t)r[L.off_d + 2 * j] | ((uint32_t)r[L.off_d + 2 * j + 1] << 8);
    } else if constexpr (FMT == kQ5_0) {
        b.p = r + 16 * j;
        b.qh = r + L.off_qh + 4 * j;
        b.d16 = (uint32_t)r[L.off_d + 2 * j] | ((uint32_t)r[L.off_d + 2 * j + 1] << 8);
    } else if constexpr (FMT == kQ4_K) {
        b.p = r + 144 * j;
    } else {
        b.p = r + 208 * j;
        b.d16 = (uint32_t)r[L.off_d + 2 * j] | ((uint32_t)r[L.off_d + 2 * j + 1] << 8);
    }
    return b;
}

template <uint32_t FMT>
__device__ __forceinline__ BlockRef ref_raw(const uint8_t *blk)
{
    BlockRef b;
    b.qh = nullptr;
    b.d16 = 0;
    if constexpr (FMT == kQ8_0) {
        b.d16 = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8);
        b.p = blk + 2;
    } else if constexpr (FMT == kQ5_0) {
        b.d16 = (uint32_t)blk[0] | ((uint32_t)blk[1] << 8);
        b.qh = blk + 2;
        b.p = blk + 6;
    } else if constexpr (FMT == kQ4_K) {
        b.p = blk;
    } else {
        b.p = blk;
        b.d16 = (uint32_t)blk[208] | ((uint32_t)blk[209] << 8);
    }
    return b;
}

template <uint32_t FMT>
__global__ void dequant_layout_kernel(Layout L, const uint8_t *__restrict__ w, float *__restrict__ out)
{
    constexpr int BE = (FMT == kQ8_0 || FMT == kQ5_0) ? 32 : 256;
    const uint64_t total = (uint64_t)L.rows * L.cols;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = e / (uint64_t)L.cols;
        const int col = (int)(e % (uint64_t)L.cols);
        const BlockRef b = ref_layout<FMT>(L, w, row, col / BE);
        out[e] = dequant_value<FMT>(b, col % BE);
    }
}

template <uint32_t FMT>
__global__ void dequant_raw_kernel(const uint8_t *__restrict__ raw, uint64_t nblocks, float *__restrict__ out)
{
    constexpr int BE = (FMT == kQ8_0 || FMT == kQ5_0) ? 32 : 256;
    constexpr int BB = (FMT == kQ8_0) ? 34 : (FMT == kQ5_0) ? 22 : (FMT == kQ4_K) ? 144 : 210;
    const uint64_t total = nblocks * BE;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < total;
         e += (uint64_t)gridDim.x * blockDim.x) {
        const BlockRef b = ref_raw<FMT>(raw + (e / BE) * BB);
        out[e] = dequant_value<FMT>(b, (int)(e % BE));
    }
}

// ------------------------------------------------------ launch helpers

int sm_count()
{
    static int count = 0;
    if (count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (count <= 0) count = 148;
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

template <typename K>
cudaError_t prepare(K kernel, size_t smem, int *blocks_per_sm)
{
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (*blocks_per_sm < 1) return cudaErrorInvalidConfiguration;
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
    constexpr int rows_per_pass = (kThreads / TPT) * R;
    long long grid = (long long)sm_count() * occ;
    long long useful = ((long long)L.rows + rows_per_pass - 1) / rows_per_pass;
    if (grid > useful) grid = useful;
    if (am && grid > kMaxArgmaxCtas) grid = kMaxArgmaxCtas;
    if (grid < 1) grid = 1;
    ArgmaxOut a = am ? *am : ArgmaxOut{nullptr, nullptr, 0};
    kernel<<<(unsigned)grid, kThreads, smem, s>>>(L, w, x, y, a, am ? 1 : 0);
    return cudaGetLastError();
}

template <uint32_t FMT, int R>
cudaError_t gemv_pick_tpt(const Layout &L, const uint8_t *w, const float *x, float *y,
                          const ArgmaxOut *am, cudaStream_t s)
{
    const int C = Chunk<FMT>::per_row(L.cols);
    if (C <= 16) return gemv_go<FMT, 16, R>(L, w, x, y, am, s);
    if (C <= 32) return gemv_go<FMT, 32, R>(L, w, x, y, am, s);
    if (C <= 64) return gemv_go<FMT, 64, R>(L, w, x, y, am, s);
    if (C <= 128) return gemv_go<FMT, 128, R>(L, w, x, y, am, s);
    return gemv_go<FMT, 256, R>(L, w, x, y, am, s);
}

template <uint32_t FMT>
cudaError_t gemv_fmt(const Layout &L, const uint8_t *w, const float *x, float *y, const ArgmaxOut *am,
                     cudaStream_t s)
{
    // Few rows per CTA -> smaller row tiles keep every group busy.
    const long long rows_per_cta = (long long)L.rows / (2LL * sm_count());
    const int C = Chunk<FMT>::per_row(L.cols);
    const int tpt = C <= 16 ? 16 : C <= 32 ? 32 : C <= 64 ? 64 : C <= 128 ? 128 : 256;
    const int groups = kThreads / tpt;
    if (rows_per_cta < 4LL * groups) return gemv_pick_tpt<FMT, 2>(L, w, x, y, am, s);
    return gemv_pick_tpt<FMT, 4>(L, w, x, y, am, s);
}

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
    constexpr int rows_per_pass = kThreads / TPT;
    long long grid = (long long)sm_count() * occ;
    long long useful = ((long long)L.rows + rows_per_pass - 1) / rows_per_pass;
    if (grid > useful) grid = useful;
    if (grid < 1) grid = 1;
    for (int p0 = 0; p0 < batch; p0 += np_max) {
        const int np = batch - p0 < np_max ? batch - p0 : np_max;
        kernel<<<(unsigned)grid, kThreads, xb * np, s>>>(L, w, X + (size_t)p0 * L.cols, np,
                                                         Y + (size_t)p0 * L.rows);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

template <uint32_t FMT>
cudaError_t matmul_fmt(const Layout &L, const uint8_t *w, const float *X, int batch, float *Y,
                       cudaStream_t s)
{
    const int C = Chunk<FMT>::per_row(L.cols);
    if (C <= 16) return matmul_go<FMT, 16>(L, w, X, batch, Y, s);
    if (C <= 32) return matmul_go<FMT, 32>(L, w, X, batch, Y, s);
    return matmul_go<FMT, 64>(L, w, X, batch, Y, s);
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
        L.off_d = 32 * nb;
        L.row_stride = L.off_d + pad16(2 * nb);
        break;
    case kQ5_0:
        L.off_qh = 16 * nb;
        L.off_d = L.off_qh + pad16(4 * nb);
        L.row_stride = L.off_d + pad16(2 * nb);
        break;
    case kQ4_K:
        L.row_stride = 144ull * nb;
        break;
    default:
        L.off_d = 208 * nb;
        L.row_stride = L.off_d + pad16(2 * nb);
        break;
    }
    *out = L;
    return true;
}

cudaError_t launch_repack(const Layout &L, const uint8_t *raw, uint8_t *dst, cudaStream_t s)
{
    cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)L.rows * L.row_stride, s);
    if (e != cudaSuccess) return e;
    const uint64_t nblocks = (uint64_t)L.rows * L.nb;
    repack_kernel<<<grid_for(nblocks, kThreads), kThreads, 0, s>>>(L, raw, dst);
    return cudaGetLastError();
}

cudaError_t launch_dequant_layout(const Layout &L, const uint8_t *w, float *out, cudaStream_t s)
{
    const unsigned g = grid_for((uint64_t)L.rows * L.cols, kThreads);
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

cudaError_t launch_argmax(const float *logits, int n, const ArgmaxOut &am, cudaStream_t s)
{
    unsigned g = grid_for((uint64_t)n, kThreads * 4);
    if (g > (unsigned)kMaxArgmaxCtas) g = kMaxArgmaxCtas;
    argmax_kernel<<<g, kThreads, 0, s>>>(logits, n, am);
    return cudaGetLastError();
}

}  // namespace qmv
