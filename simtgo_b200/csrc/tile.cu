// tile.cu -- the tile track (package tile): graph recording (tile/tile.go),
// lowering to one fused program (tile/codegen.go) and running it
// (tile/run.go), with no run-time compiler.
//
// The reference renders each graph as CUDA C and compiles it with NVRTC per
// distinct graph (tile/run.go:40). Here the graph is lowered on the host to a
// short register program that travels in the kernel's parameter block, and
// ONE precompiled sm_100a kernel interprets it:
//  * a block works on chunks of 2048 elements, a thread on 8 consecutive
//    ones; values live in 8 register slots of 8 floats each;
//  * the program is copied to shared memory once per block; every
//    instruction is warp-uniform and dispatches on its kind, then on its
//    destination (and source) slot, so all slot indices are compile-time and
//    values never leave registers;
//  * every input is read from HBM once: a block's chunk of each input (plus
//    the windows' halo) is brought into shared memory by cp.async.bulk, in
//    as many stages as the block's share of the SM's shared memory holds, so
//    later chunks stream in while one is interpreted (inputs that are not
//    16-byte aligned are loaded directly); the result is written once with
//    16-byte streaming stores -- 4 bytes per input and 4 bytes out per
//    element, one pass over HBM;
//  * a windowed (FIR) node is evaluated as in tile/codegen.go:80-108: its
//    signal sub-expression is run by the same interpreter over the chunk
//    plus a halo of taps-1 (zero outside the signal), staged in shared
//    memory, then each thread forms fma(h[k], tile, acc) in k order for its
//    8 outputs from three 16-byte shared loads per 4 taps.
// Every operation is rounded on its own (Scale = k*x, Add, Mul, Sqrt
// correctly rounded, Abs exact, Hypot = gpu.Hypot), so the fused program and
// the stepwise one (one launch per node, tile/run.go:89) agree bit for bit.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "exact.cuh"
#include "tma.cuh"

using namespace sgd;

namespace tilek {

constexpr int kSlots = 8;
constexpr int kV = 8;  // elements per thread per instruction
constexpr int kThreads = 256;
constexpr int kChunk = kThreads * kV;  // elements per block iteration
constexpr int kMaxCode = 1024;
constexpr int kMaxIn = 32;
constexpr int kMaxFir = 8;
constexpr int kMaxTaps = SIMTGO_TILE_MAX_TAPS;
constexpr int kTileF = kChunk + kMaxTaps + 16;  // staged floats per window node
constexpr int kMaxStages = 16;                 // input stages in flight (bulk mode)

// An instruction word is kind << 6 | d << 3 | s: the operation, the
// destination slot and the source slot. The interpreter dispatches on the
// kind (12 cases), then on d or on (d, s) (8 or 64 cases): small dense
// switches with compile-time slot indices in every case.
enum Op : uint16_t {
    OP_END = 0,
    OP_LOAD,    // r[d] = input aux
    OP_STORE,   // out = r[d]
    OP_STAGE,   // window tile = r[d]
    OP_FIRACC,  // r[d] = window aux accumulated at the thread's positions
    OP_SCALE,   // r[d] = imm * r[d]
    OP_SQRT,    // r[d] = sqrt(r[d])
    OP_ABS,     // r[d] = |r[d]|
    OP_MOV,     // r[d] = r[s]
    OP_ADD,     // r[d] = r[d] + r[s]
    OP_MUL,     // r[d] = r[d] * r[s]
    OP_HYPOT,   // r[d] = hypot(r[d], r[s])
    OP_KINDS,
};
__host__ __device__ constexpr uint16_t enc(int op, int d, int s = 0) {
    return (uint16_t)((op << 6) | (d << 3) | s);
}

struct Insn {
    uint16_t code;
    uint16_t aux;
    float imm;
};

struct FirDesc {
    int32_t start;  // pc of the staging program
    int32_t taps;
    float h[kMaxTaps];  // the coefficients travel in the parameter block
};

struct Program {
    int32_t main_start;
    int32_t n_fir;
    int32_t n_in;
    int32_t n_code;
    FirDesc fir[kMaxFir];
    const float* in[kMaxIn];  // element 0 of each input; in[k][i] is valid for i in [-halo, n)
    Insn code[kMaxCode];
};

// Eight consecutive elements of one value.
struct V8 {
    float4 a, b;
};

// The program as the interpreter reads it: copied once per block from the
// parameter bank into shared memory, where a warp-uniform word is one
// broadcast load (the parameter bank, indexed by a run-time pc, is not).
// Layout: code[code_cap] | in[n_in] | fir[n_fir] (start, taps), 16-byte
// rounded.
__host__ __device__ constexpr int meta_code_cap(int n_code) { return (n_code + 2) & ~1; }
__host__ __device__ constexpr int meta_bytes(int n_code, int n_in, int n_fir) {
    return ((meta_code_cap(n_code) * 8 + n_in * 8 + n_fir * 8) + 15) & ~15;
}

struct Exec {
    const Insn* code;         // shared copy of Program::code
    const float* const* in;   // shared copy of Program::in
    const int2* fir;          // shared (start, taps) of each window node
    int64_t p0;     // first of the thread's 8 positions
    int64_t n;      // shard length
    int64_t halo;   // positions [-halo, n) are valid
    bool vec;       // all inputs and out are 16-byte aligned
    float* out;
    float* stage;   // STAGE target (tile + offset of p0)
    const float* taps_s;
    const float* tiles;
    int64_t cb;     // chunk base (for FIRACC)
    // Inputs staged in shared memory (bulk-copy mode), or null: position p
    // of input k is sin[k * sstride + (p - sorg)].
    const float* sin;
    int64_t sorg;
    int32_t sstride;
};

__device__ __forceinline__ float lane_of(const V8& v, int e) {
    switch (e) {
        case 0: return v.a.x;
        case 1: return v.a.y;
        case 2: return v.a.z;
        case 3: return v.a.w;
        case 4: return v.b.x;
        case 5: return v.b.y;
        case 6: return v.b.z;
        default: return v.b.w;
    }
}

// Lanes of v at positions outside [-halo, n) replaced by 0.
__device__ __forceinline__ V8 mask_outside(V8 v, const Exec& x) {
    const int64_t p = x.p0;
    if (p >= -x.halo && p + 7 < x.n) return v;
    float f[8] = {v.a.x, v.a.y, v.a.z, v.a.w, v.b.x, v.b.y, v.b.z, v.b.w};
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (!(p + e >= -x.halo && p + e < x.n)) f[e] = 0.0f;
    return {make_float4(f[0], f[1], f[2], f[3]), make_float4(f[4], f[5], f[6], f[7])};
}

__device__ __forceinline__ V8 load_pos(int k, const Exec& x) {
    const int64_t p = x.p0;
    if (x.sin) {
        // Shared memory: two aligned 16-byte loads; lanes outside the signal
        // read whatever the buffer holds there and are zeroed.
        const float* s = x.sin + (int64_t)k * x.sstride + (p - x.sorg);
        V8 v = {*reinterpret_cast<const float4*>(s), *reinterpret_cast<const float4*>(s + 4)};
        return mask_outside(v, x);
    }
    const float* base = x.in[k];
    if (x.vec && p >= -x.halo && p + 7 < x.n)
        return {ld_stream_f4(base + p), ld_stream_f4(base + p + 4)};
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; e++) f[e] = (p + e >= -x.halo && p + e < x.n) ? base[p + e] : 0.0f;
    return {make_float4(f[0], f[1], f[2], f[3]), make_float4(f[4], f[5], f[6], f[7])};
}

__device__ __forceinline__ void store_pos(const V8& v, const Exec& x) {
    const int64_t p = x.p0;
    if (x.vec && p + 7 < x.n) {
        st_stream_f4(x.out + p, v.a);
        st_stream_f4(x.out + p + 4, v.b);
        return;
    }
#pragma unroll
    for (int e = 0; e < 8; e++)
        if (p + e < x.n) x.out[p + e] = lane_of(v, e);
}

__device__ __forceinline__ void stage_pos(const V8& v, const Exec& x) {
    const V8 s = mask_outside(v, x);
    *reinterpret_cast<float4*>(x.stage) = s.a;
    *reinterpret_cast<float4*>(x.stage + 4) = s.b;
}

// Window start of node f for chunk cb: 16-byte aligned, 4 floats of slack
// below the first halo sample.
__device__ __forceinline__ int64_t tile_start(int64_t cb, int taps) {
    return ((cb - (taps - 1)) & ~int64_t(3)) - 4;
}

// The window accumulation of one thread's 8 outputs, out of line so that the
// interpreter's FIRACC cases stay small. tile/h: the window's staged samples
// and taps in shared memory; q0: the tile index of the thread's first
// position (a multiple of 4). Output e at tap k0+u reads tile index
// q0 + e - k0 - u = w[4 + e - u] with w = tile + q0 - k0 - 4.
__device__ __noinline__ V8 fir_acc_window(const float* tile, const float* h, int taps, int q0) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; e++) acc[e] = 0.0f;
    for (int k0 = 0; k0 < taps; k0 += 4) {
        const float* w = tile + (q0 - k0 - 4);
        const float4 w0 = *reinterpret_cast<const float4*>(w);
        const float4 w1 = *reinterpret_cast<const float4*>(w + 4);
        const float4 w2 = *reinterpret_cast<const float4*>(w + 8);
        const float wv[12] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w,
                              w2.x, w2.y, w2.z, w2.w};
        const float4 hk = *reinterpret_cast<const float4*>(h + k0);
        const float hv[4] = {hk.x, hk.y, hk.z, hk.w};
        const int nk = min(4, taps - k0);
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (u < nk)
#pragma unroll
                for (int e = 0; e < 8; e++) acc[e] = __fmaf_rn(hv[u], wv[4 + e - u], acc[e]);
    }
    return {make_float4(acc[0], acc[1], acc[2], acc[3]),
            make_float4(acc[4], acc[5], acc[6], acc[7])};
}

__device__ __forceinline__ V8 fir_acc(int f, const Exec& x) {
    const int taps = x.fir[f].y;
    return fir_acc_window(x.tiles + f * kTileF, x.taps_s + f * kMaxTaps, taps,
                          (int)(x.p0 - tile_start(x.cb, taps)));
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                       __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) {
    return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z),
                       __fmul_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_scale(float k, float4 a) {
    return make_float4(__fmul_rn(k, a.x), __fmul_rn(k, a.y), __fmul_rn(k, a.z),
                       __fmul_rn(k, a.w));
}
__device__ __forceinline__ float4 f4_sqrt(float4 a) {
    return make_float4(__fsqrt_rn(a.x), __fsqrt_rn(a.y), __fsqrt_rn(a.z), __fsqrt_rn(a.w));
}
__device__ __forceinline__ float4 f4_abs(float4 a) {
    return make_float4(fabsf(a.x), fabsf(a.y), fabsf(a.z), fabsf(a.w));
}
__device__ __forceinline__ V8 v_add(const V8& p, const V8& q) {
    return {f4_add(p.a, q.a), f4_add(p.b, q.b)};
}
__device__ __forceinline__ V8 v_mul(const V8& p, const V8& q) {
    return {f4_mul(p.a, q.a), f4_mul(p.b, q.b)};
}
__device__ __forceinline__ V8 v_scale(float k, const V8& p) {
    return {f4_scale(k, p.a), f4_scale(k, p.b)};
}
__device__ __noinline__ V8 v_sqrt(V8 p) { return {f4_sqrt(p.a), f4_sqrt(p.b)}; }
__device__ __forceinline__ V8 v_abs(const V8& p) { return {f4_abs(p.a), f4_abs(p.b)}; }
// Out of line: 64 interpreter cases call it.
__device__ __noinline__ V8 v_hypot(V8 p, V8 q) {
    return {make_float4(hypot_go(p.a.x, q.a.x), hypot_go(p.a.y, q.a.y), hypot_go(p.a.z, q.a.z),
                        hypot_go(p.a.w, q.a.w)),
            make_float4(hypot_go(p.b.x, q.b.x), hypot_go(p.b.y, q.b.y), hypot_go(p.b.z, q.b.z),
                        hypot_go(p.b.w, q.b.w))};
}

#define SG_D8(M) M(0) M(1) M(2) M(3) M(4) M(5) M(6) M(7)
#define SG_S8(M, D) M(D, 0) M(D, 1) M(D, 2) M(D, 3) M(D, 4) M(D, 5) M(D, 6) M(D, 7)
#define SG_DS64(M)                                                                         \
    SG_S8(M, 0) SG_S8(M, 1) SG_S8(M, 2) SG_S8(M, 3) SG_S8(M, 4) SG_S8(M, 5) SG_S8(M, 6) \
        SG_S8(M, 7)

#define C_SET(D) \
    case D:      \
        r[D] = v;  \
        break;
#define C_GET(D) \
    case D:      \
        v = r[D];  \
        break;
#define C_SCALE(D)                      \
    case D:                             \
        r[D] = v_scale(in.imm, r[D]);   \
        break;
#define C_SQRT(D)           \
    case D:                 \
        r[D] = v_sqrt(r[D]); \
        break;
#define C_ABS(D)            \
    case D:                 \
        r[D] = v_abs(r[D]); \
        break;
#define C_MOV(D, S)     \
    case 8 * D + S:     \
        r[D] = r[S];    \
        break;
#define C_ADD(D, S)               \
    case 8 * D + S:               \
        r[D] = v_add(r[D], r[S]); \
        break;
#define C_MUL(D, S)               \
    case 8 * D + S:               \
        r[D] = v_mul(r[D], r[S]); \
        break;
#define C_HYPOT(D, S)               \
    case 8 * D + S:                 \
        r[D] = v_hypot(r[D], r[S]); \
        break;

// Runs the program from pc until OP_END for the thread's 8 positions.
// Inlined at its one call site in k_tile, so x stays in registers. The next
// word is loaded while this one executes (the copy holds one word past END).
__device__ __forceinline__ void interpret(int pc, const Exec& x) {
    V8 r[kSlots];
    const V8 zero = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
    for (int i = 0; i < kSlots; i++) r[i] = zero;
    Insn next = x.code[pc];
    for (;;) {
        const Insn in = next;
        next = x.code[++pc];
        const int op = in.code >> 6, d = (in.code >> 3) & 7, ds = in.code & 63;
        V8 v = zero;
        switch (op) {
            case OP_LOAD:
                v = load_pos(in.aux, x);
                switch (d) { SG_D8(C_SET) }
                break;
            case OP_FIRACC:
                v = fir_acc(in.aux, x);
                switch (d) { SG_D8(C_SET) }
                break;
            case OP_STORE:
                switch (d) { SG_D8(C_GET) }
                store_pos(v, x);
                break;
            case OP_STAGE:
                switch (d) { SG_D8(C_GET) }
                stage_pos(v, x);
                break;
            case OP_SCALE:
                switch (d) { SG_D8(C_SCALE) }
                break;
            case OP_SQRT:
                switch (d) { SG_D8(C_SQRT) }
                break;
            case OP_ABS:
                switch (d) { SG_D8(C_ABS) }
                break;
            case OP_MOV:
                switch (ds) { SG_DS64(C_MOV) }
                break;
            case OP_ADD:
                switch (ds) { SG_DS64(C_ADD) }
                break;
            case OP_MUL:
                switch (ds) { SG_DS64(C_MUL) }
                break;
            case OP_HYPOT:
                switch (ds) { SG_DS64(C_HYPOT) }
                break;
            default:
                return;  // OP_END
        }
    }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

struct ChunkSpan {
    int64_t org, lo, len4, hi;  // buffer origin, copied [lo, lo+len4), valid [lo, hi)
};

__device__ __forceinline__ ChunkSpan chunk_span(int64_t cb, int hs, int64_t n, int64_t halo) {
    ChunkSpan s;
    s.org = cb - hs;
    s.lo = max(s.org, -halo);
    s.hi = min(cb + (int64_t)kChunk, n);
    s.len4 = s.hi > s.lo ? ((s.hi - s.lo) & ~int64_t(3)) : 0;
    return s;
}

// Bulk-copy mode (BULK): the chunk's inputs (positions [cb - hs, cb + kChunk),
// clipped to the signal) travel HBM -> shared memory by cp.async.bulk, one
// copy per input, in `nst` stages that complete on per-stage mbarriers, so
// nst-1 chunks stream in while one is interpreted. Requires every input
// 16-byte aligned and halo = 0 mod 4.
template <bool BULK>
__global__ void __launch_bounds__(kThreads) k_tile(const __grid_constant__ Program P,
                                                   float* __restrict__ out, int64_t n,
                                                   int64_t halo, bool vec, int32_t hs,
                                                   int32_t nst, uint32_t* wd) {
    __shared__ __align__(8) uint64_t bars[kMaxStages];
    extern __shared__ float4 sm4[];
    const int code_cap = meta_code_cap(P.n_code);
    Insn* code_s = reinterpret_cast<Insn*>(sm4);
    const float** in_s = reinterpret_cast<const float**>(code_s + code_cap);
    int2* fir_s = reinterpret_cast<int2*>(in_s + P.n_in);
    float* sm = reinterpret_cast<float*>(sm4) + meta_bytes(P.n_code, P.n_in, P.n_fir) / 4;
    float* taps_s = sm;                        // n_fir x kMaxTaps
    float* tiles = sm + P.n_fir * kMaxTaps;    // n_fir x kTileF
    float* stages = tiles + P.n_fir * kTileF;  // nst x n_in x sstride (bulk mode)
    // Each input's buffer: the chunk and its halo, plus 8 floats that the
    // last staging task's whole 8-float loads may touch past the chunk.
    const int32_t sstride = kChunk + hs + 8;
    const int64_t stage_floats = (int64_t)P.n_in * sstride;
    const int tid = threadIdx.x;
    const int64_t nchunks = (n + kChunk - 1) / kChunk;
    for (int i = tid; i < code_cap; i += kThreads)
        code_s[i] = i < P.n_code ? P.code[i] : Insn{enc(OP_END, 0), 0, 0.0f};
    for (int k = tid; k < P.n_in; k += kThreads) in_s[k] = P.in[k];
    for (int f = tid; f < P.n_fir; f += kThreads) fir_s[f] = make_int2(P.fir[f].start, P.fir[f].taps);
    for (int f = 0; f < P.n_fir; f++)
        for (int k = tid; k < kMaxTaps; k += kThreads)
            taps_s[f * kMaxTaps + k] = P.fir[f].h[k];  // zero past taps

    auto issue = [&](int64_t c, int s) {
        const ChunkSpan sp = chunk_span(c * kChunk, hs, n, halo);
        mbar_arrive_expect_tx(&bars[s], (uint32_t)(sp.len4 * 4 * P.n_in));
        if (sp.len4 > 0)
            for (int k = 0; k < P.n_in; k++)
                bulk_g2s(stages + s * stage_floats + (int64_t)k * sstride + (sp.lo - sp.org),
                         in_s[k] + sp.lo, (uint32_t)(sp.len4 * 4), &bars[s]);
    };
    if (BULK) {
        if (tid == 0) {
            for (int s = 0; s < nst; s++) mbar_init(&bars[s], 1);
            fence_mbar_init();
        }
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < nst; s++) {
                const int64_t c = blockIdx.x + (int64_t)s * gridDim.x;
                if (c < nchunks) issue(c, s);
            }
    }
    __syncthreads();

    Exec x;
    x.code = code_s;
    x.in = in_s;
    x.fir = fir_s;
    x.n = n;
    x.halo = halo;
    x.vec = vec;
    x.out = out;
    x.taps_s = taps_s;
    x.tiles = tiles;
    x.sin = nullptr;
    x.sorg = 0;
    x.sstride = sstride;
    int it = 0;
    for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x, it++) {
        const int64_t cb = c * kChunk;
        x.cb = cb;
        if (BULK) {
            const int s = it % nst;
            if (!mbar_wait(&bars[s], (uint32_t)((it / nst) & 1), wd)) return;
            const ChunkSpan sp = chunk_span(cb, hs, n, halo);
            float* buf = stages + s * stage_floats;
            // The last 0-3 samples of a ragged signal are not a whole 16-byte
            // unit: plain loads.
            const int64_t tail = sp.hi - (sp.lo + sp.len4);
            if (tail > 0 && tid < P.n_in * 4) {
                const int k = tid / 4, e = tid % 4;
                const int64_t pos = sp.lo + sp.len4 + e;
                if (e < tail) buf[(int64_t)k * sstride + (pos - sp.org)] = in_s[k][pos];
            }
            __syncthreads();
            x.sin = buf;
            x.sorg = sp.org;
        }
        // Jobs f = 0 .. n_fir-1 stage window f's signal over its span (the
        // chunk plus the halo); job n_fir is the main program over the
        // chunk. One loop, so the interpreter is inlined exactly once.
        const int nf = P.n_fir;
        for (int f = 0; f <= nf; f++) {
            int64_t base, span;
            int pc;
            float* st = tiles;
            if (f < nf) {
                const int2 fd = fir_s[f];
                base = tile_start(cb, fd.y);
                span = cb + kChunk - base;
                pc = fd.x;
                st = tiles + f * kTileF;
            } else {
                base = cb;
                span = min((int64_t)kChunk, n - cb);
                pc = P.main_start;
            }
            for (int64_t off = kV * tid; off < span; off += kV * kThreads) {
                x.p0 = base + off;
                x.stage = st + off;
                interpret(pc, x);
            }
            if (f + 1 == nf) __syncthreads();  // windows staged before main reads them
        }
        if (BULK) {
            // Every thread is done with this stage (and with the tiles);
            // order those generic accesses before the next bulk copy into it.
            fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) {
                const int64_t cn = c + (int64_t)nst * gridDim.x;
                if (cn < nchunks) issue(cn, it % nst);
            }
        } else if (P.n_fir > 0) {
            __syncthreads();
        }
    }
}

}  // namespace tilek

// ============================================================================
// Host side: the recorded graph (tile/tile.go) and its lowering.
// ============================================================================

namespace {

enum Kind { K_INPUT = 0, K_SCALE, K_ADD, K_MUL, K_SQRT, K_ABS, K_HYPOT, K_FIR };

struct Node {
    Kind kind;
    int32_t n;
    int a = -1, b = -1;
    float scale = 0.0f;
    const float* host = nullptr;  // K_INPUT with host data
    const float* dev = nullptr;   // K_INPUT with device data
    std::vector<float> taps;      // K_INPUT that holds a FIR's coefficients (copied)
    bool is_taps = false;
};

}  // namespace

struct simtgo_tile_graph {
    std::vector<Node> nodes;
    std::string err;
};

namespace {

using tilek::Insn;
using tilek::Program;

void latch(simtgo_tile_graph* g, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void latch(simtgo_tile_graph* g, const char* fmt, ...) {
    if (!g->err.empty()) return;  // the first error is kept (tile/tile.go:78-82)
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g->err = std::string("tile: ") + buf;
}

bool valid(const simtgo_tile_graph* g, simtgo_tensor t) {
    return g && t >= 0 && (size_t)t < g->nodes.size();
}

simtgo_tensor add_node(simtgo_tile_graph* g, Node nd) {
    g->nodes.push_back(std::move(nd));
    return (simtgo_tensor)(g->nodes.size() - 1);
}

bool contains_fir(const simtgo_tile_graph* g, int id) {
    const Node& n = g->nodes[id];
    if (n.kind == K_FIR) return true;
    if (n.a >= 0 && contains_fir(g, n.a)) return true;
    if (n.b >= 0 && contains_fir(g, n.b)) return true;
    return false;
}

// postorder (tile/codegen.go:135-144): dependencies first, each node once.
void postorder(const simtgo_tile_graph* g, int id, std::vector<int>& out, std::vector<char>& seen,
               bool stop_at_fir) {
    if (seen[id]) return;
    seen[id] = 1;
    const Node& n = g->nodes[id];
    if (!(stop_at_fir && n.kind == K_FIR)) {
        if (n.a >= 0) postorder(g, n.a, out, seen, stop_at_fir);
        if (n.b >= 0) postorder(g, n.b, out, seen, stop_at_fir);
    }
    out.push_back(id);
}

struct Lowered {
    Program prog;
    std::vector<int> in_nodes;   // data input node ids, in prog.in order
    std::vector<int> fir_nodes;  // window node ids, in prog.fir order
    std::vector<int> param_of;   // reference parameter index pK of each data input
};

// Emits one program computing `root` (main: root's value, window nodes read
// from their tiles; staging: a window's signal, stopped at nothing since a
// signal contains no window). Register slots are assigned linearly over the
// postorder; a slot is reused as soon as its value has no uses left.
int emit_program(const simtgo_tile_graph* g, int root, bool main, Lowered& L, bool hoist,
                 std::unordered_map<int, int>& input_index,
                 std::unordered_map<int, int>& fir_index, std::vector<Insn>& code) {
    std::vector<int> order;
    std::vector<char> seen(g->nodes.size(), 0);
    postorder(g, root, order, seen, main);
    std::vector<int> uses(g->nodes.size(), 0);
    for (int id : order) {
        const Node& n = g->nodes[id];
        if (main && n.kind == K_FIR) continue;
        if (n.kind == K_INPUT) continue;
        if (n.a >= 0) uses[n.a]++;
        if (n.b >= 0) uses[n.b]++;
    }
    std::vector<int> slot(g->nodes.size(), -1);
    bool free_slot[tilek::kSlots];
    for (bool& f : free_slot) f = true;
    auto alloc = [&]() -> int {
        for (int s = 0; s < tilek::kSlots; s++)
            if (free_slot[s]) {
                free_slot[s] = false;
                return s;
            }
        return -1;
    };
    auto push = [&](uint16_t c, uint16_t aux = 0, float imm = 0.0f) {
        code.push_back(Insn{c, aux, imm});
    };
    auto load = [&](int id) -> int {
        int s = alloc();
        if (s < 0) return -1;
        auto it = input_index.find(id);
        int k;
        if (it == input_index.end()) {
            k = (int)L.in_nodes.size();
            if (k >= tilek::kMaxIn) return -2;
            input_index[id] = k;
            L.in_nodes.push_back(id);
        } else {
            k = it->second;
        }
        push(tilek::enc(tilek::OP_LOAD, s), (uint16_t)k);
        slot[id] = s;
        return s;
    };
    if (hoist)
        for (int id : order)
            if (g->nodes[id].kind == K_INPUT && slot[id] < 0)
                if (load(id) < 0) return -1;
    auto need = [&](int id) -> int {
        if (slot[id] >= 0) return slot[id];
        return load(id);  // not hoisted
    };
    auto release = [&](int id) {
        if (--uses[id] == 0 && slot[id] >= 0) free_slot[slot[id]] = true;
    };
    for (int id : order) {
        const Node& n = g->nodes[id];
        if (n.kind == K_INPUT) {
            if (id == root && need(id) < 0) return -1;
            continue;
        }
        if (main && n.kind == K_FIR) {
            int d = alloc();
            if (d < 0) return -1;
            auto it = fir_index.find(id);
            if (it == fir_index.end()) return -3;
            push(tilek::enc(tilek::OP_FIRACC, d), (uint16_t)it->second);
            slot[id] = d;
            continue;
        }
        if (n.kind == K_FIR) return -3;  // a window inside a signal is refused at build
        const bool unary = (n.kind == K_SCALE || n.kind == K_SQRT || n.kind == K_ABS);
        const int sa = need(n.a);
        if (sa < 0) return -1;
        int d;
        if (unary) {
            if (uses[n.a] == 1) {
                d = sa;
                slot[n.a] = -1;
                uses[n.a] = 0;
            } else {
                d = alloc();
                if (d < 0) return -1;
                push(tilek::enc(tilek::OP_MOV, d, sa));
                release(n.a);
            }
            if (n.kind == K_SCALE) push(tilek::enc(tilek::OP_SCALE, d), 0, n.scale);
            if (n.kind == K_SQRT) push(tilek::enc(tilek::OP_SQRT, d));
            if (n.kind == K_ABS) push(tilek::enc(tilek::OP_ABS, d));
        } else {
            const int sb = need(n.b);
            if (sb < 0) return -1;
            const int bop = n.kind == K_ADD   ? tilek::OP_ADD
                            : n.kind == K_MUL ? tilek::OP_MUL
                                              : tilek::OP_HYPOT;
            if (n.a == n.b) {
                if (uses[n.a] == 2) {
                    d = sa;
                    slot[n.a] = -1;
                    uses[n.a] = 0;
                } else {
                    d = alloc();
                    if (d < 0) return -1;
                    push(tilek::enc(tilek::OP_MOV, d, sa));
                    release(n.a);
                    release(n.a);
                }
                push(tilek::enc(bop, d, d));
            } else if (uses[n.a] == 1) {
                d = sa;
                slot[n.a] = -1;
                uses[n.a] = 0;
                push(tilek::enc(bop, d, sb));
                release(n.b);
            } else if (uses[n.b] == 1) {
                // Add, Mul and Hypot are commutative bit for bit.
                d = sb;
                slot[n.b] = -1;
                uses[n.b] = 0;
                push(tilek::enc(bop, d, sa));
                release(n.a);
            } else {
                d = alloc();
                if (d < 0) return -1;
                push(tilek::enc(tilek::OP_MOV, d, sa));
                push(tilek::enc(bop, d, sb));
                release(n.a);
                release(n.b);
            }
        }
        slot[id] = d;
    }
    push(tilek::enc(main ? tilek::OP_STORE : tilek::OP_STAGE, slot[root]));
    push(tilek::enc(tilek::OP_END, 0));
    return 0;
}

// Lowers the graph rooted at t. Returns 0 or a status (message recorded).
int lower(const simtgo_tile_graph* g, int root, Lowered& L) {
    memset(&L.prog, 0, sizeof L.prog);
    L.in_nodes.clear();
    L.fir_nodes.clear();
    L.param_of.clear();
    // The reference's parameter numbering: every input node, taps included,
    // in postorder (tile/codegen.go:24-35).
    {
        std::vector<int> order;
        std::vector<char> seen(g->nodes.size(), 0);
        postorder(g, root, order, seen, false);
        int p = 0;
        std::unordered_map<int, int> pidx;
        for (int id : order)
            if (g->nodes[id].kind == K_INPUT) pidx[id] = p++;
        for (int id : order)
            if (g->nodes[id].kind == K_FIR) L.fir_nodes.push_back(id);
        L.param_of.resize(g->nodes.size(), -1);
        for (auto& kv : pidx) L.param_of[kv.first] = kv.second;
    }
    if ((int)L.fir_nodes.size() > tilek::kMaxFir)
        return sg::fail(SIMTGO_ESIZE, "tile: %zu windowed operations; the fused kernel stages at most %d",
                        L.fir_nodes.size(), tilek::kMaxFir);
    std::unordered_map<int, int> fir_index;
    for (size_t i = 0; i < L.fir_nodes.size(); i++) fir_index[L.fir_nodes[i]] = (int)i;
    for (int hoist = 1; hoist >= 0; hoist--) {
        std::vector<Insn> code;
        std::unordered_map<int, int> input_index;
        L.in_nodes.clear();
        int rc = 0;
        for (size_t f = 0; f < L.fir_nodes.size() && rc == 0; f++) {
            const Node& fn = g->nodes[L.fir_nodes[f]];
            L.prog.fir[f].start = (int32_t)code.size();
            const std::vector<float>& h = g->nodes[fn.b].taps;
            L.prog.fir[f].taps = (int32_t)h.size();
            for (size_t k = 0; k < h.size(); k++) L.prog.fir[f].h[k] = h[k];
            rc = emit_program(g, fn.a, false, L, hoist, input_index, fir_index, code);
        }
        if (rc == 0) {
            L.prog.main_start = (int32_t)code.size();
            rc = emit_program(g, root, true, L, hoist, input_index, fir_index, code);
        }
        if (rc == -2)
            return sg::fail(SIMTGO_ESIZE, "tile: more than %d distinct inputs", tilek::kMaxIn);
        if (rc == -3) return sg::fail(SIMTGO_EGRAPH, "tile: a windowed operation inside a window");
        if (rc == -1) continue;  // out of slots: retry without hoisting the loads
        if (code.size() > (size_t)tilek::kMaxCode)
            return sg::fail(SIMTGO_ESIZE, "tile: the program has %zu instructions (max %d)",
                            code.size(), tilek::kMaxCode);
        memcpy(L.prog.code, code.data(), code.size() * sizeof(Insn));
        L.prog.n_code = (int32_t)code.size();
        L.prog.n_fir = (int32_t)L.fir_nodes.size();
        L.prog.n_in = (int32_t)L.in_nodes.size();
        return 0;
    }
    return sg::fail(SIMTGO_ESIZE,
                    "tile: the graph keeps more than %d values live at once; materialise part of it",
                    tilek::kSlots);
}

// Launches a lowered program. dev_in[k] = device data of L.in_nodes[k] (halo
// elements first).
int launch_program(Lowered& L, const std::vector<const float*>& dev_in, float* out, int64_t n,
                   int64_t halo, cudaStream_t s) {
    const sg::DevInfo* d;
    int rc;
    if ((rc = sg::current_device(&d))) return rc;
    if (n <= 0) return 0;
    bool vec = sg::aligned16(out);
    bool in_aligned = true;
    for (size_t k = 0; k < dev_in.size(); k++) {
        L.prog.in[k] = dev_in[k];  // element 0 of the shard; [-halo, 0) precede it
        in_aligned = in_aligned && sg::aligned16(L.prog.in[k]);
    }
    vec = vec && in_aligned;
    // Samples a chunk's windows reach below it: the widest window's taps-1,
    // rounded up to 16 bytes, plus tile_start's 4 floats of slack.
    int32_t hs = 0;
    for (int f = 0; f < L.prog.n_fir; f++)
        hs = std::max<int32_t>(hs, (L.prog.fir[f].taps - 1 + 3) / 4 * 4 + 4);
    const size_t base_smem =
        tilek::meta_bytes(L.prog.n_code, L.prog.n_in, L.prog.n_fir) +
        (size_t)L.prog.n_fir * (tilek::kMaxTaps + tilek::kTileF) * sizeof(float);
    const size_t stage_bytes =
        (size_t)L.prog.n_in * (tilek::kChunk + hs + 8) * sizeof(float);
    // Both instantiations may take up to the opt-in maximum of dynamic
    // shared memory (less 1 KB for the static mbarriers); the stage count
    // below decides how much they use.
    const int dyn_max = d->max_smem_optin - 1024;
    static std::atomic<uint64_t> configured{0};
    const uint64_t dev_bit = 1ull << (d->device & 63);
    if (!(configured.load() & dev_bit)) {
        for (auto k : {tilek::k_tile<true>, tilek::k_tile<false>}) {
            rc = sg::cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      dyn_max),
                                 "cudaFuncSetAttribute(tile)");
            if (rc) return rc;
        }
        configured.fetch_or(dev_bit);
    }
    // Input stages: registers bound the blocks per SM; the stages then take
    // that block's share of the SM's shared memory (2..kMaxStages chunks of
    // every input in flight), since HBM latency x bandwidth per SM is tens
    // of KB that must be outstanding at once.
    int per_sm = 0;
    rc = sg::cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                             &per_sm, tilek::k_tile<true>, tilek::kThreads, base_smem),
                         "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
    if (rc) return rc;
    const int64_t share = std::min<int64_t>(dyn_max,
                                            d->smem_per_sm / std::max(1, per_sm) - 2048);
    int nst = (int)std::max<int64_t>(2, (share - (int64_t)base_smem) / (int64_t)stage_bytes);
    nst = std::min(nst, tilek::kMaxStages);
    const size_t bulk_smem = base_smem + nst * stage_bytes;
    const bool bulk = in_aligned && halo % 4 == 0 && L.prog.n_in > 0 &&
                      bulk_smem <= (size_t)dyn_max;
    const size_t smem = bulk ? bulk_smem : base_smem;
    auto kern = bulk ? tilek::k_tile<true> : tilek::k_tile<false>;
    rc = sg::cuda_status(
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, tilek::kThreads, smem),
        "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
    if (rc) return rc;
    const int64_t chunks = sg::ceil_div(n, tilek::kChunk);
    const int blocks = (int)std::max<int64_t>(
        1, std::min<int64_t>(chunks, (int64_t)d->sms * std::max(1, per_sm)));
    sg::before_launch();
    kern<<<blocks, tilek::kThreads, smem, s>>>(L.prog, out, n, halo, vec, hs, nst,
                                               sg::watchdog_device_ptr());
    return sg::launch_status("tile");
}

// A device allocation owned by one materialisation. Move-only: a container
// that relocates it must not free the memory it still refers to.
struct DevBuf {
    float* p = nullptr;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p) { o.p = nullptr; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        std::swap(p, o.p);
        return *this;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
};

int upload(const float* host, int64_t n, DevBuf& b) {
    int rc = sg::cuda_status(cudaMalloc(&b.p, std::max<int64_t>(n, 1) * sizeof(float)),
                             "cudaMalloc");
    if (rc) return rc;
    if (n > 0)
        rc = sg::cuda_status(cudaMemcpy(b.p, host, n * sizeof(float), cudaMemcpyHostToDevice),
                             "upload");
    return rc;
}

// tile/alias.go:42-78: the output may not overlap an input it reads.
int check_out_alias(const Lowered& L, const simtgo_tile_graph* g, const float* out, int64_t n,
                    const std::vector<const float*>& dev_in, int64_t halo) {
    const uintptr_t o0 = (uintptr_t)out, o1 = o0 + (uintptr_t)n * 4;
    for (size_t k = 0; k < dev_in.size(); k++) {
        const Node& nd = g->nodes[L.in_nodes[k]];
        const uintptr_t i0 = (uintptr_t)(dev_in[k] - halo), i1 = (uintptr_t)(dev_in[k] + nd.n);
        if (o0 >= i1 || i0 >= o1) continue;
        return sg::fail(SIMTGO_EALIAS,
                        "tile: the output buffer overlaps input p%d, which the kernel reads while "
                        "it writes out; the generated kernel declares every pointer __restrict__, "
                        "which promises that they do not overlap",
                        L.param_of[L.in_nodes[k]]);
    }
    return 0;
}

// Runs the fused program for root with inputs resolved by `resolve`
// (node id -> device pointer).
template <class Resolve>
int run_fused(const simtgo_tile_graph* g, int root, float* out, int64_t n, int64_t halo,
              cudaStream_t s, Resolve resolve, bool check_alias) {
    Lowered L;
    int rc = lower(g, root, L);
    if (rc) return rc;
    std::vector<const float*> dev_in;
    for (int id : L.in_nodes) {
        const float* p = resolve(id);
        if (!p) return sg::fail(SIMTGO_EARG, "tile: input node %d has no device data", id);
        dev_in.push_back(p);
    }
    if (check_alias && (rc = check_out_alias(L, g, out, n, dev_in, halo))) return rc;
    return launch_program(L, dev_in, out, n, halo, s);
}

}  // namespace

extern "C" {

simtgo_tile_graph* simtgo_tile_new(void) { return new simtgo_tile_graph(); }

void simtgo_tile_free(simtgo_tile_graph* g) { delete g; }

simtgo_tensor simtgo_tile_input(simtgo_tile_graph* g, const float* host, int32_t n) {
    if (!g) return -1;
    if (n < 0) latch(g, "Input: negative length %d", n);
    if (n > 0 && !host) latch(g, "Input: null data for %d elements", n);
    Node nd;
    nd.kind = K_INPUT;
    nd.n = std::max(n, 0);
    nd.host = host;
    return add_node(g, std::move(nd));
}

simtgo_tensor simtgo_tile_input_device(simtgo_tile_graph* g, const float* dev, int32_t n) {
    if (!g) return -1;
    if (n < 0) latch(g, "Input: negative length %d", n);
    if (n > 0 && !dev) latch(g, "Input: null device data for %d elements", n);
    Node nd;
    nd.kind = K_INPUT;
    nd.n = std::max(n, 0);
    nd.dev = dev;
    return add_node(g, std::move(nd));
}

static simtgo_tensor binary(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b, Kind k,
                            const char* name) {
    if (!g) return -1;
    if (!valid(g, a) || !valid(g, b)) {
        latch(g, "%s: operands come from different graphs", name);
        return a;
    }
    if (g->nodes[a].n != g->nodes[b].n) {
        latch(g, "%s: length %d does not match %d", name, g->nodes[a].n, g->nodes[b].n);
        return a;
    }
    Node nd;
    nd.kind = k;
    nd.n = g->nodes[a].n;
    nd.a = a;
    nd.b = b;
    return add_node(g, std::move(nd));
}

simtgo_tensor simtgo_tile_add(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b) {
    return binary(g, a, b, K_ADD, "Add");
}
simtgo_tensor simtgo_tile_mul(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b) {
    return binary(g, a, b, K_MUL, "Mul");
}
simtgo_tensor simtgo_tile_hypot(simtgo_tile_graph* g, simtgo_tensor a, simtgo_tensor b) {
    return binary(g, a, b, K_HYPOT, "Hypot");
}

static simtgo_tensor unary(simtgo_tile_graph* g, simtgo_tensor a, Kind k, float scale,
                           const char* name) {
    if (!g) return -1;
    if (!valid(g, a)) {
        latch(g, "%s: the operand is not a tensor of this graph", name);
        return a;
    }
    Node nd;
    nd.kind = k;
    nd.n = g->nodes[a].n;
    nd.a = a;
    nd.scale = scale;
    return add_node(g, std::move(nd));
}

simtgo_tensor simtgo_tile_scale(simtgo_tile_graph* g, simtgo_tensor a, float k) {
    return unary(g, a, K_SCALE, k, "Scale");
}
simtgo_tensor simtgo_tile_sqrt(simtgo_tile_graph* g, simtgo_tensor a) {
    return unary(g, a, K_SQRT, 0, "Sqrt");
}
simtgo_tensor simtgo_tile_abs(simtgo_tile_graph* g, simtgo_tensor a) {
    return unary(g, a, K_ABS, 0, "Abs");
}

simtgo_tensor simtgo_tile_fir(simtgo_tile_graph* g, simtgo_tensor a, const float* h,
                              int32_t taps) {
    if (!g) return -1;
    if (!valid(g, a)) {
        latch(g, "FIR: the operand is not a tensor of this graph");
        return a;
    }
    if (taps <= 0 || taps > SIMTGO_TILE_MAX_TAPS) {
        latch(g, "FIR: %d taps is outside 1..%d", taps, SIMTGO_TILE_MAX_TAPS);
        return a;
    }
    if (!h) {
        latch(g, "FIR: null coefficients");
        return a;
    }
    if (contains_fir(g, a)) {
        latch(g, "FIR: chaining windowed operations is not supported; materialise the first one");
        return a;
    }
    Node t;
    t.kind = K_INPUT;
    t.n = taps;
    t.taps.assign(h, h + taps);
    t.is_taps = true;
    const simtgo_tensor tid = add_node(g, std::move(t));
    Node f;
    f.kind = K_FIR;
    f.n = g->nodes[a].n;
    f.a = a;
    f.b = tid;
    return add_node(g, std::move(f));
}

int32_t simtgo_tile_len(const simtgo_tile_graph* g, simtgo_tensor t) {
    return valid(g, t) ? g->nodes[t].n : -1;
}

int simtgo_tile_err(const simtgo_tile_graph* g) {
    if (!g) return SIMTGO_ENULL;
    return g->err.empty() ? SIMTGO_OK : SIMTGO_EGRAPH;
}

const char* simtgo_tile_err_string(const simtgo_tile_graph* g) {
    return g ? g->err.c_str() : "tile: null graph";
}

int simtgo_tile_program_size(simtgo_tile_graph* g, simtgo_tensor t, int32_t* n_instructions,
                             int32_t* n_inputs, int32_t* n_windows) {
    sg::clear_error();
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    if (!g->err.empty()) return sg::fail(SIMTGO_EGRAPH, "%s", g->err.c_str());
    if (!valid(g, t)) return sg::fail(SIMTGO_EARG, "tile: unknown tensor %d", t);
    Lowered L;
    int rc = lower(g, t, L);
    if (rc) return rc;
    if (n_instructions) *n_instructions = L.prog.n_code;
    if (n_inputs) *n_inputs = L.prog.n_in;
    if (n_windows) *n_windows = L.prog.n_fir;
    return 0;
}

// The listing of a lowered program, one instruction per line:
//   "window <f> taps <T>" / "main" section headers, then
//   "<pc> load r<d> in<k>", "scale r<d> <k as %a>", "sqrt r<d>", "abs r<d>",
//   "mov r<d> r<s>", "add|mul|hypot r<d> r<s>", "firacc r<d> w<f>",
//   "store r<s>", "stage r<s>", "end".
static std::string listing(const simtgo_tile_graph* g, const Lowered& L) {
    std::string s;
    char line[160];
    snprintf(line, sizeof line, "; simtgo_b200 tile program: %d instructions, %d inputs, %d windows\n",
             L.prog.n_code, L.prog.n_in, L.prog.n_fir);
    s += line;
    for (int k = 0; k < L.prog.n_in; k++) {
        snprintf(line, sizeof line, "; in%d = node %d (p%d)\n", k, L.in_nodes[k],
                 L.param_of[L.in_nodes[k]]);
        s += line;
    }
    for (int pc = 0; pc < L.prog.n_code; pc++) {
        for (int f = 0; f < L.prog.n_fir; f++)
            if (L.prog.fir[f].start == pc) {
                snprintf(line, sizeof line, "window %d taps %d node %d\n", f, L.prog.fir[f].taps,
                         L.fir_nodes[f]);
                s += line;
            }
        if (pc == L.prog.main_start) s += "main\n";
        const Insn& in = L.prog.code[pc];
        using namespace tilek;
        const int op = in.code >> 6, d = (in.code >> 3) & 7, sl = in.code & 7;
        switch (op) {
            case OP_END: snprintf(line, sizeof line, "%d end\n", pc); break;
            case OP_LOAD: snprintf(line, sizeof line, "%d load r%d in%d\n", pc, d, in.aux); break;
            case OP_STORE: snprintf(line, sizeof line, "%d store r%d\n", pc, d); break;
            case OP_STAGE: snprintf(line, sizeof line, "%d stage r%d\n", pc, d); break;
            case OP_FIRACC:
                snprintf(line, sizeof line, "%d firacc r%d w%d\n", pc, d, in.aux);
                break;
            case OP_SCALE:
                snprintf(line, sizeof line, "%d scale r%d %a\n", pc, d, (double)in.imm);
                break;
            case OP_SQRT: snprintf(line, sizeof line, "%d sqrt r%d\n", pc, d); break;
            case OP_ABS: snprintf(line, sizeof line, "%d abs r%d\n", pc, d); break;
            default: {
                const char* name = op == OP_MOV   ? "mov"
                                   : op == OP_ADD ? "add"
                                   : op == OP_MUL ? "mul"
                                                  : "hypot";
                snprintf(line, sizeof line, "%d %s r%d r%d\n", pc, name, d, sl);
            }
        }
        s += line;
    }
    (void)g;
    return s;
}

static int check_run(simtgo_tile_graph* g, simtgo_tensor t, int32_t out_len) {
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    if (!g->err.empty()) return sg::fail(SIMTGO_EGRAPH, "%s", g->err.c_str());
    if (!valid(g, t)) return sg::fail(SIMTGO_EARG, "tile: unknown tensor %d", t);
    if (out_len != g->nodes[t].n)
        return sg::fail(SIMTGO_ELENGTH, "tile: the output holds %d elements, the tensor has %d",
                        out_len, g->nodes[t].n);
    return 0;
}

int32_t simtgo_tile_source(simtgo_tile_graph* g, simtgo_tensor t, char* buf, int32_t cap) {
    sg::clear_error();
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    if (!g->err.empty()) return sg::fail(SIMTGO_EGRAPH, "%s", g->err.c_str());
    if (!valid(g, t)) return sg::fail(SIMTGO_EARG, "tile: unknown tensor %d", t);
    Lowered L;
    int rc = lower(g, t, L);
    if (rc) return rc;
    const std::string s = listing(g, L);
    if (buf && cap > 0) {
        const size_t n = std::min<size_t>(s.size(), (size_t)cap - 1);
        memcpy(buf, s.data(), n);
        buf[n] = 0;
    }
    return (int32_t)s.size() + 1;
}

int simtgo_tile_materialize(simtgo_tile_graph* g, simtgo_tensor t, float* host_out,
                            int32_t out_len) {
    sg::clear_error();
    int rc;
    if ((rc = check_run(g, t, out_len))) return rc;
    const int64_t n = out_len;
    if (n == 0) return 0;
    if (!host_out) return sg::fail(SIMTGO_ENULL, "tile: null output");
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    std::vector<DevBuf> owned;
    std::unordered_map<int, const float*> uploaded;
    DevBuf out;
    if ((rc = sg::cuda_status(cudaMalloc(&out.p, n * sizeof(float)), "cudaMalloc"))) return rc;
    int err = 0;
    auto resolve = [&](int id) -> const float* {
        const Node& nd = g->nodes[id];
        if (nd.dev) return nd.dev;
        auto it = uploaded.find(id);
        if (it != uploaded.end()) return it->second;
        owned.emplace_back();
        if (int r = upload(nd.host, nd.n, owned.back())) {
            err = r;
            return nullptr;
        }
        uploaded[id] = owned.back().p;
        return owned.back().p;
    };
    rc = run_fused(g, t, out.p, n, 0, 0, resolve, true);
    if (err) return err;
    if (rc) return rc;
    return sg::cuda_status(cudaMemcpy(host_out, out.p, n * sizeof(float), cudaMemcpyDeviceToHost),
                           "download");
}

int simtgo_tile_materialize_stepwise(simtgo_tile_graph* g, simtgo_tensor t, float* host_out,
                                     int32_t out_len, int32_t* launches) {
    sg::clear_error();
    int rc;
    if (launches) *launches = 0;
    if ((rc = check_run(g, t, out_len))) return rc;
    const int64_t n = out_len;
    if (n > 0 && !host_out) return sg::fail(SIMTGO_ENULL, "tile: null output");
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    // tile/run.go:113 step: every node materialised into a device buffer of
    // its own, through a one-operation graph over the buffers of its arguments.
    std::vector<DevBuf> owned;
    std::unordered_map<int, const float*> buf;
    std::vector<int> order;
    std::vector<char> seen(g->nodes.size(), 0);
    postorder(g, t, order, seen, false);
    int count = 0;
    for (int id : order) {
        const Node& nd = g->nodes[id];
        if (nd.kind == K_INPUT) {
            if (nd.is_taps) continue;
            if (nd.dev) {
                buf[id] = nd.dev;
            } else {
                owned.emplace_back();
                if ((rc = upload(nd.host, nd.n, owned.back()))) return rc;
                buf[id] = owned.back().p;
            }
            continue;
        }
        simtgo_tile_graph one;
        const int a = simtgo_tile_input_device(&one, buf[nd.a], g->nodes[nd.a].n);
        int r;
        if (nd.kind == K_FIR) {
            const Node& tp = g->nodes[nd.b];
            r = simtgo_tile_fir(&one, a, tp.taps.data(), (int32_t)tp.taps.size());
        } else if (nd.kind == K_SCALE) {
            r = simtgo_tile_scale(&one, a, nd.scale);
        } else if (nd.kind == K_SQRT) {
            r = simtgo_tile_sqrt(&one, a);
        } else if (nd.kind == K_ABS) {
            r = simtgo_tile_abs(&one, a);
        } else {
            // A node feeding both operands is one buffer read twice (tile/run.go:122-127).
            const int b = nd.b == nd.a ? a
                                       : simtgo_tile_input_device(&one, buf[nd.b], g->nodes[nd.b].n);
            r = nd.kind == K_ADD   ? simtgo_tile_add(&one, a, b)
                : nd.kind == K_MUL ? simtgo_tile_mul(&one, a, b)
                                   : simtgo_tile_hypot(&one, a, b);
        }
        owned.emplace_back();
        if ((rc = sg::cuda_status(cudaMalloc(&owned.back().p, std::max<int64_t>(nd.n, 1) * 4),
                                  "cudaMalloc")))
            return rc;
        float* outp = owned.back().p;
        auto resolve = [&](int nid) -> const float* { return one.nodes[nid].dev; };
        rc = run_fused(&one, r, outp, nd.n, 0, 0, resolve, true);
        count++;
        if (launches) *launches = count;
        if (rc) return rc;
        buf[id] = outp;
    }
    if (n == 0) return 0;
    if ((rc = sg::cuda_status(cudaDeviceSynchronize(), "stepwise"))) return rc;
    return sg::cuda_status(
        cudaMemcpy(host_out, buf[t], n * sizeof(float), cudaMemcpyDeviceToHost), "download");
}

int simtgo_tile_run_shard(simtgo_tile_graph* g, simtgo_tensor t, float* dev_out,
                          int32_t out_len, int32_t halo, void* stream) {
    sg::clear_error();
    int rc;
    if ((rc = check_run(g, t, out_len))) return rc;
    if (halo < 0) return sg::fail(SIMTGO_EARG, "tile: negative halo");
    if (out_len == 0) return 0;
    if (!dev_out) return sg::fail(SIMTGO_ENULL, "tile: null output");
    auto resolve = [&](int id) -> const float* { return g->nodes[id].dev; };
    return run_fused(g, t, dev_out, out_len, halo, (cudaStream_t)stream, resolve, true);
}

int simtgo_tile_run(simtgo_tile_graph* g, simtgo_tensor t, float* dev_out, int32_t out_len,
                    void* stream) {
    return simtgo_tile_run_shard(g, t, dev_out, out_len, 0, stream);
}

}  // extern "C"

// ---- the stepwise run without allocation ------------------------------------
// Scratch for simtgo_tile_run_stepwise_noalloc: the values of the graph's
// intermediate nodes. A fixed array in the module, so every GPU that loads
// the library holds these 16 MiB until the process exits.
namespace {
constexpr int64_t kNoAllocFloats = SIMTGO_TILE_NOALLOC_SCRATCH_FLOATS;
constexpr int64_t kNoAllocAlign = 64;  // floats: each node's region starts 256-byte aligned
}  // namespace
static __device__ __align__(256) float g_stepwise_scratch[kNoAllocFloats];

namespace {
std::mutex g_scratch_mu;
float* g_scratch_ptr[64];

// The device address of g_stepwise_scratch on the current device. Host code
// may not use the symbol itself as an address (it names a host-side
// stand-in); the runtime resolves it once per device, with that device
// current.
int stepwise_scratch(float** out) {
    int dev = -1;
    int rc = sg::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return sg::fail(SIMTGO_EDEVICE, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        rc = sg::cuda_status(cudaGetSymbolAddress(&p, g_stepwise_scratch),
                             "cudaGetSymbolAddress(stepwise scratch)");
        if (rc) return rc;
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return 0;
}
}  // namespace

extern "C" int simtgo_tile_run_stepwise_noalloc(simtgo_tile_graph* g, simtgo_tensor t,
                                                float* dev_out, int32_t out_len, void* stream) {
    sg::clear_error();
    int rc;
    if ((rc = check_run(g, t, out_len))) return rc;
    if (out_len == 0) return 0;
    if (!dev_out) return sg::fail(SIMTGO_ENULL, "tile: null output");
    std::vector<int> order;
    std::vector<char> seen(g->nodes.size(), 0);
    postorder(g, t, order, seen, false);
    // Every value must already be on the device, and every intermediate node
    // gets its own region of the scratch array: nothing is allocated.
    std::vector<int64_t> region(g->nodes.size(), -1);
    int64_t used = 0;
    for (int id : order) {
        const Node& nd = g->nodes[id];
        if (nd.kind == K_INPUT) {
            if (!nd.is_taps && !nd.dev)
                return sg::fail(SIMTGO_EARG,
                                "tile: the allocation-free run needs device-resident inputs "
                                "(node %d is host data)",
                                id);
            continue;
        }
        if (id == t) continue;  // the root is written straight to dev_out
        region[id] = used;
        used += (nd.n + kNoAllocAlign - 1) / kNoAllocAlign * kNoAllocAlign;
    }
    if (used > kNoAllocFloats)
        return sg::fail(SIMTGO_ESIZE,
                        "tile: the allocation-free stepwise run needs %lld floats of scratch for "
                        "the graph's intermediate values; its fixed scratch holds %lld (16 MiB)",
                        (long long)used, (long long)kNoAllocFloats);
    float* scratch = nullptr;
    if ((rc = stepwise_scratch(&scratch))) return rc;
    auto value = [&](int id) -> const float* {
        return g->nodes[id].kind == K_INPUT ? g->nodes[id].dev : scratch + region[id];
    };
    for (int id : order) {
        const Node& nd = g->nodes[id];
        if (nd.kind == K_INPUT) continue;
        simtgo_tile_graph one;
        const int a = simtgo_tile_input_device(&one, value(nd.a), g->nodes[nd.a].n);
        int r;
        if (nd.kind == K_FIR) {
            const Node& tp = g->nodes[nd.b];
            r = simtgo_tile_fir(&one, a, tp.taps.data(), (int32_t)tp.taps.size());
        } else if (nd.kind == K_SCALE) {
            r = simtgo_tile_scale(&one, a, nd.scale);
        } else if (nd.kind == K_SQRT) {
            r = simtgo_tile_sqrt(&one, a);
        } else if (nd.kind == K_ABS) {
            r = simtgo_tile_abs(&one, a);
        } else {
            const int b = nd.b == nd.a ? a : simtgo_tile_input_device(&one, value(nd.b), g->nodes[nd.b].n);
            r = nd.kind == K_ADD   ? simtgo_tile_add(&one, a, b)
                : nd.kind == K_MUL ? simtgo_tile_mul(&one, a, b)
                                   : simtgo_tile_hypot(&one, a, b);
        }
        float* target = id == t ? dev_out : scratch + region[id];
        auto resolve = [&](int nid) -> const float* { return one.nodes[nid].dev; };
        rc = run_fused(&one, r, target, nd.n, 0, (cudaStream_t)stream, resolve, true);
        if (rc) return rc;
    }
    return 0;
}

extern "C" {

}  // extern "C"
