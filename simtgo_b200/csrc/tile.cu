// tile.cu -- the tile track (package tile): graph recording (tile/tile.go),
// lowering to one fused program (tile/codegen.go) and running it
// (tile/run.go), with no run-time compiler.
//
// The reference renders each graph as CUDA C and compiles it with NVRTC per
// distinct graph (tile/run.go:40). Here the graph is lowered on the host to a
// short program for an accumulator machine that travels in the kernel's
// parameter block, and ONE precompiled sm_100a kernel interprets it:
//  * a block works on chunks of 2048 elements; a thread owns 2 float4 groups
//    of each chunk (groups t and t + 256, so a warp's 16-byte shared-memory
//    accesses are consecutive and conflict-free) held in an accumulator of
//    8 registers;
//  * every instruction combines the accumulator with at most one operand in
//    shared memory -- a staged input, a temporary, or a window's staged
//    signal -- so the interpreter dispatches on the operation alone and the
//    operand is an address, not a register index: a dispatch costs a few
//    instructions for 8 elements, and a thread needs few registers, so many
//    warps hide the latency;
//  * every input is read from HBM once: a block's chunk of each input (plus
//    the windows' halo) is brought into shared memory by cp.async.bulk, in
//    as many stages as the block's share of the SM's shared memory holds, so
//    later chunks stream in while one is interpreted (inputs that are not
//    16-byte aligned are copied by the threads); the result is written once
//    with 16-byte streaming stores -- 4 bytes per input and 4 bytes out per
//    element, one pass over HBM;
//  * a windowed (FIR) node is evaluated as in tile/codegen.go:80-108: its
//    signal sub-expression is run by the same interpreter over the chunk
//    plus a halo of taps-1 (zero outside the signal), staged in shared
//    memory, then each thread forms fma(h[k], tile, acc) in k order for its
//    8 outputs, one new 16-byte shared load per group per 4 taps. The staged
//    signal also serves the main program wherever it uses that node;
//  * with chained windows (an opt-in; the reference rejects a FIR of an
//    expression holding a FIR) a window's signal program reads the windows
//    inside it, which are staged first;
//  * a reduction of the graph (Sum, Min, Max, ArgMax; the reference has
//    none) consumes the main program's values in the same pass: each warp
//    reduces its part of a chunk in a fixed tree to one partial in HBM, and
//    small level kernels finish the tree.
// Every operation is rounded on its own (Scale = k*x, Add, Mul, Sqrt
// correctly rounded, Abs exact, Hypot = gpu.Hypot), so the fused program and
// the stepwise one (one launch per node, tile/run.go:89) agree bit for bit.
// Add, Mul and Hypot are commutative bit for bit, which lets the lowering
// keep either operand in the accumulator.
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

constexpr int kThreads = 256;
// Float4 groups per thread (the template parameter G): 2 for graphs with
// windows or Hypot, 4 (kGWide) for the others, whose dispatch and chunk
// costs then spread over twice the elements (eight chained Muls measured
// 0.57 -> 0.76 of HBM; Hypot's registers make it slower there).
constexpr int kG = 2;
constexpr int kGWide = 4;
__host__ __device__ constexpr int chunk_of(int G) { return kThreads * 4 * G; }
// 2048: the chunk of G = 2 (every window's tile is laid out for it) and the
// block of the reduction trees, whatever G the interpreter runs with.
constexpr int kChunk = chunk_of(kG);
constexpr int kChunk4 = kChunk / 4;
constexpr int kMaxCode = 1024;
constexpr int kMaxIn = 32;
constexpr int kMaxFir = 8;
constexpr int kMaxTmp = 8;
constexpr int kMaxTaps = SIMTGO_TILE_MAX_TAPS;
// Samples a chunk's window reaches below it: taps-1 rounded up to 16 bytes,
// plus 4 of slack so that the first 16-byte window load stays in the tile.
__host__ __device__ constexpr int window_reach(int taps) { return (taps - 1 + 3) / 4 * 4 + 4; }
// Staged floats of a window's tile: its head, the chunk and 4 of slack.
__host__ __device__ constexpr int tile_floats(int head) { return kChunk + head + 4; }
constexpr int kMaxStages = 16;
// FirDesc.taps flag: a later window's staging reads this window's tile, so
// the block synchronises after staging it (chained windows).
constexpr int32_t kSyncAfter = 1 << 8;

// Steps of the accumulator machine. A is the accumulator (the thread's
// 8 elements), M an operand in shared memory. The lowering emits these one
// by one; a device instruction fuses a run of them (below).
enum Op : uint8_t {
    OP_END = 0,
    OP_LDA,     // A = M
    OP_STA,     // M = A (a temporary)
    OP_ADD,     // A = A + M
    OP_MUL,     // A = A * M
    OP_HYPOT,   // A = hypot(A, M)
    OP_SCALE,   // A = imm * A
    OP_SQRT,    // A = sqrt(A)
    OP_ABS,     // A = |A|
    OP_FIRACC,  // A = window b accumulated at the thread's positions
    OP_STAGE,   // window's tile = A (zero outside the signal)
    OP_STORE,   // out = A
    OP_KINDS,
};
// A device instruction is one dispatch doing, in order: [A = M(a)] if
// F_LOADA; the operation op (ADD/MUL/HYPOT with operand M(b), SCALE, SQRT,
// ABS, FIRACC of window b; OP_END: none); [M(d) = A] if F_STA; [tile of
// window d = A] if F_STAGE; [out = A] if F_STORE; return if F_END.
constexpr uint8_t F_LOADA = 1;
constexpr uint8_t F_IN_A = 2;   // M(a) is a staged input: a is relative to the current stage
constexpr uint8_t F_IN_B = 4;   // M(b) likewise
constexpr uint8_t F_SELF = 8;   // M(b) is A itself (x op x)
constexpr uint8_t F_STA = 16;
constexpr uint8_t F_STAGE = 32;
constexpr uint8_t F_STORE = 64;
constexpr uint8_t F_END = 128;

struct Insn {
    uint8_t op;
    uint8_t flags;
    uint16_t a;  // F_LOADA operand: float4 offset in shared memory (or input index, DIRECT)
    uint16_t b;  // binary operand likewise, or the FIRACC window
    uint16_t d;  // F_STA temporary (float4 offset) or F_STAGE window
    float imm;   // SCALE factor
    uint32_t pad;
};
static_assert(sizeof(Insn) == 16, "one 16-byte shared load per instruction");

struct FirDesc {
    int32_t start;  // pc of the staging program
    int32_t taps;   // the taps, | kSyncAfter when a later window reads this one
    int32_t head;   // positions the tile holds below the chunk (a multiple of 4)
    int32_t tile4;  // float4 offset of the window's tile in shared memory
    float h[kMaxTaps];  // the coefficients travel in the parameter block
};

// Reductions (SIMTGO_TILE_SUM ..): the main program's value is reduced
// instead of stored.
enum Reduce : int32_t { RED_NONE = -1, RED_SUM = 0, RED_MIN = 1, RED_MAX = 2, RED_ARGMAX = 3 };

struct Program {
    int32_t main_start;
    int32_t reduce;  // RED_NONE, or the reduction of the main program's value
    int32_t n_fir;
    int32_t n_in;
    int32_t n_code;
    FirDesc fir[kMaxFir];
    const float* in[kMaxIn];  // element 0 of each input; in[k][i] is valid for i in [-halo, n)
    Insn code[kMaxCode];
};

// The program as the interpreter reads it: copied once per block from the
// parameter bank into shared memory, where a warp-uniform word is one
// broadcast load. Layout: code[code_cap] (the program and one END) |
// fir[n_fir] (start, taps | flags, head, tile4) | in[n_in], 16-byte rounded.
__host__ __device__ constexpr int meta_code_cap(int n_code) { return n_code + 1; }
__host__ __device__ constexpr int meta_bytes(int n_code, int n_in, int n_fir) {
    return ((meta_code_cap(n_code) * 16 + n_in * 8 + n_fir * 16) + 15) & ~15;
}

// One run of a program over kChunk (or, for a window's halo, fewer)
// positions.
struct Run {
    int32_t sh_in;   // added to F_IN operands: the stage and the run's position
    int32_t sh_st;   // added to STAGE destinations (the run's offset in the tile)
    int32_t woff4;   // (run position - chunk position) / 4: where FIRACC reads a tile
    uint32_t gm;     // which of the thread's groups take part
    int64_t p0;      // position of the run's element 0
    bool edge;       // some positions of the run lie outside [-halo, n)
};

struct Ctx {
    float4* S;               // dynamic shared memory
    const float* taps_s;     // n_fir x kMaxTaps coefficients, zero past taps
    const int4* fir;         // shared (start, taps | flags, head, tile4)
    const float* const* in;  // shared copy of Program::in
    float* out;
    int64_t n, halo;
    bool vec;                // out is 16-byte aligned
    bool in_vec;             // every input is 16-byte aligned
};

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
__device__ __forceinline__ float4 f4_hypot(float4 a, float4 b) {
    return make_float4(hypot_go(a.x, b.x), hypot_go(a.y, b.y), hypot_go(a.z, b.z),
                       hypot_go(a.w, b.w));
}
__device__ __forceinline__ float f4_get(const float4& v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// The window accumulation for the thread's groups: output j of group k sits
// at tile index b_k + j, b_k = 4 (t + 256 k + woff4) + head, and takes
// fma(h[i], tile[b_k + j - i], acc) for i = 0 .. taps-1 in order. With
// W = tile[b_k - i0 - 4 .. b_k - i0 + 3] for taps i0 .. i0+3, the sample of
// output j at tap i0+u is W[4 + j - u]; the upper half of W is the lower
// half of the previous step, so each step loads one new float4 per group.
// Four taps (hv[0..nk-1]) on the 4 outputs of one group, with
// w = tile[b - i0 - 4 .. b - i0 + 3] given as its halves lo, hi.
template <bool PART>
__device__ __forceinline__ void fir_step(float (&acc)[4], const float4& lo, const float4& hi,
                                         const float (&hv)[4], int nk) {
    const float w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int u = 0; u < 4; u++)
        if (!PART || u < nk)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[j] = __fmaf_rn(hv[u], w[4 + j - u], acc[j]);
}

template <int G>
__device__ __forceinline__ void fir_acc(float4 (&A)[G], const Ctx& c, int f, int woff4) {
    const int4 fd = c.fir[f];
    const int taps = fd.y & (kSyncAfter - 1);
    const float4* h4 = reinterpret_cast<const float4*>(c.taps_s + f * kMaxTaps);
    // Group k's window float4 at tap i0 (a multiple of 4): tw[k][-i0/4].
    const float4* tw = c.S + fd.w + threadIdx.x + fd.z / 4 + woff4;
    float acc[G][4];
    float4 hi[G];
#pragma unroll
    for (int k = 0; k < G; k++) {
#pragma unroll
        for (int j = 0; j < 4; j++) acc[k][j] = 0.0f;
        hi[k] = tw[kThreads * k];
    }
    // Whole steps of 8 taps, two window loads per group, no predicates.
    int i0 = 0;
    for (; i0 + 8 <= taps; i0 += 8) {
        const float4 ha = h4[i0 / 4], hb = h4[i0 / 4 + 1];
        const float hva[4] = {ha.x, ha.y, ha.z, ha.w}, hvb[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int k = 0; k < G; k++) {
            const float4 m = tw[kThreads * k - i0 / 4 - 1];
            const float4 lo = tw[kThreads * k - i0 / 4 - 2];
            fir_step<false>(acc[k], m, hi[k], hva, 4);
            fir_step<false>(acc[k], lo, m, hvb, 4);
            hi[k] = lo;
        }
    }
    // The last 1-7 taps, 4 at a time.
    for (; i0 < taps; i0 += 4) {
        const float4 hk = h4[i0 / 4];
        const float hv[4] = {hk.x, hk.y, hk.z, hk.w};
        const int nk = min(4, taps - i0);
#pragma unroll
        for (int k = 0; k < G; k++) {
            const float4 lo = tw[kThreads * k - i0 / 4 - 1];
            fir_step<true>(acc[k], lo, hi[k], hv, nk);
            hi[k] = lo;
        }
    }
#pragma unroll
    for (int k = 0; k < G; k++) A[k] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
}

// Positions p .. p+3 of input b read from HBM (DIRECT mode), 0 outside
// [-halo, n).
__device__ __forceinline__ float4 gload4(const float* b, int64_t p, const Ctx& c) {
    if (p >= -c.halo && p + 3 < c.n)
        return c.in_vec ? ld_stream_f4(b + p) : make_float4(b[p], b[p + 1], b[p + 2], b[p + 3]);
    float f[4];
#pragma unroll
    for (int j = 0; j < 4; j++) f[j] = (p + j >= -c.halo && p + j < c.n) ? b[p + j] : 0.0f;
    return make_float4(f[0], f[1], f[2], f[3]);
}

// Zeroes the lanes of v whose positions (p .. p+3) lie outside [-halo, n).
__device__ __forceinline__ float4 mask_outside(float4 v, int64_t p, const Ctx& c) {
    if (p >= -c.halo && p + 3 < c.n) return v;
    float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++)
        if (!(p + j >= -c.halo && p + j < c.n)) f[j] = 0.0f;
    return make_float4(f[0], f[1], f[2], f[3]);
}

// Runs the program from pc until an instruction with F_END, leaving the
// last value in A (which a reduction consumes). Inlined into
// k_tile twice: FULL for runs where all of the thread's groups take part
// (the chunk), and the general form for a window's head run. (Loading the
// next instruction ahead measured slower: it costs more instructions than
// the shared-load latency it hides.) In DIRECT mode (BULK false) an input
// operand is read from HBM at the run's positions.
template <bool BULK, bool FULL, int G>
__device__ __forceinline__ void interpret(const Insn* code, int pc, const Ctx& c, const Run& r,
                                          float4 (&A)[G]) {
    const int t = threadIdx.x;
#pragma unroll
    for (int k = 0; k < G; k++) A[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (;;) {
        const Insn in = code[pc++];
        // Group k of operand M(x) (inactive groups: A itself, nothing is read).
        auto operand = [&](int x, bool input, int k) -> float4 {
            if (!FULL && !((r.gm >> k) & 1)) return A[k];
            if (!BULK && input) return gload4(c.in[x], r.p0 + 4 * (t + kThreads * k), c);
            return c.S[x + (input ? r.sh_in : 0) + t + kThreads * k];
        };
        if (in.flags & F_LOADA) {
#pragma unroll
            for (int k = 0; k < G; k++) A[k] = operand(in.a, in.flags & F_IN_A, k);
        }
        // The second operand of a binary operation, read inside its case.
        auto binop = [&](int k) -> float4 {
            return (in.flags & F_SELF) ? A[k] : operand(in.b, in.flags & F_IN_B, k);
        };
        switch (in.op) {
            case OP_ADD:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_add(A[k], binop(k));
                break;
            case OP_MUL:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_mul(A[k], binop(k));
                break;
            case OP_HYPOT:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_hypot(A[k], binop(k));
                break;
            case OP_SCALE:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_scale(in.imm, A[k]);
                break;
            case OP_SQRT:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_sqrt(A[k]);
                break;
            case OP_ABS:
#pragma unroll
                for (int k = 0; k < G; k++) A[k] = f4_abs(A[k]);
                break;
            case OP_FIRACC:
                fir_acc<G>(A, c, in.b, r.woff4);
                break;
            default:
                break;  // OP_END: no operation
        }
        if (in.flags & (F_STA | F_STAGE | F_STORE | F_END)) {
            if (in.flags & F_STA) {
#pragma unroll
                for (int k = 0; k < G; k++)
                    if (FULL || ((r.gm >> k) & 1)) c.S[in.d + t + kThreads * k] = A[k];
            }
            if (in.flags & F_STAGE) {
                float4* dst = c.S + c.fir[in.d].w + r.sh_st + t;
#pragma unroll
                for (int k = 0; k < G; k++)
                    if (FULL || ((r.gm >> k) & 1))
                        dst[kThreads * k] =
                            r.edge ? mask_outside(A[k], r.p0 + 4 * (t + kThreads * k), c) : A[k];
            }
            if (in.flags & F_STORE) {
#pragma unroll
                for (int k = 0; k < G; k++) {
                    const int64_t p = r.p0 + 4 * (t + kThreads * k);
                    if (c.vec && p + 3 < c.n) {
                        st_stream_f4(c.out + p, A[k]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; j++)
                            if (p + j < c.n) c.out[p + j] = f4_get(A[k], j);
                    }
                }
            }
            if (in.flags & F_END) return;
        }
    }
}

// ---- reductions ---------------------------------------------------------------
// A value and, for ARGMAX, its index. The empty identity of ARGMAX is
// (-inf, INT64_MAX): any element beats it. Every step is a template on the
// reduction, so a chunk's reduction is straight-line code.
struct RVal {
    float v;
    int64_t i;
};
constexpr int64_t kNoIndex = INT64_MAX;
constexpr uint32_t kQNaN = 0x7fc00000u;

template <int KIND>
__device__ __forceinline__ RVal red_identity() {
    if (KIND == RED_SUM) return {0.0f, 0};
    if (KIND == RED_MIN) return {__int_as_float(0x7f800000), 0};
    return {__int_as_float((int)0xff800000u), kNoIndex};
}
// Go's min and max (NaN wins, -0 < +0); NaN is returned as 0x7fc00000.
// Branch-free: fminf/fmaxf, then equal values (only zeros of opposite signs
// differ in bits) combined by OR (min: -0 wins) or AND (max: +0 wins), then
// NaN.
__device__ __forceinline__ float go_min(float a, float b) {
    float m = fminf(a, b);
    if (a == b) m = __uint_as_float(__float_as_uint(a) | __float_as_uint(b));
    return (a != a || b != b) ? __uint_as_float(kQNaN) : m;
}
__device__ __forceinline__ float go_max(float a, float b) {
    float m = fmaxf(a, b);
    if (a == b) m = __uint_as_float(__float_as_uint(a) & __float_as_uint(b));
    return (a != a || b != b) ? __uint_as_float(kQNaN) : m;
}
// ARGMAX order: NaN above everything, then value (+0 above -0), then the
// smaller index. A strict total order on distinct indices, so any tree of
// pairwise choices finds the same element. (Early returns measured faster
// here than evaluating every clause and selecting.)
__device__ __forceinline__ bool am_before(const RVal& a, const RVal& b) {
    const bool na = a.v != a.v, nb = b.v != b.v;
    if (na || nb) return na && nb ? a.i < b.i : na;
    if (a.v > b.v) return true;
    if (b.v > a.v) return false;
    const bool sa = __float_as_uint(a.v) >> 31, sb = __float_as_uint(b.v) >> 31;
    if (sa != sb) return !sa;
    return a.i < b.i;
}
template <int KIND>
__device__ __forceinline__ RVal red2(const RVal& a, const RVal& b) {
    if (KIND == RED_SUM) return {__fadd_rn(a.v, b.v), 0};
    if (KIND == RED_MIN) return {go_min(a.v, b.v), 0};
    if (KIND == RED_MAX) return {go_max(a.v, b.v), 0};
    return am_before(a, b) ? a : b;
}
// The caller's result: a NaN sum as 0x7fc00000 (NaN payloads differ by
// platform), ARGMAX's empty index as -1.
template <int KIND>
__device__ __forceinline__ RVal red_final(RVal r) {
    if (KIND == RED_SUM && r.v != r.v) r.v = __uint_as_float(kQNaN);
    if (KIND == RED_ARGMAX && r.i == kNoIndex) r.i = -1;
    return r;
}
// A thread's eight values: x[0..3] its group at 4t, x[4..7] at 1024 + 4t.
template <int KIND>
__device__ __forceinline__ RVal red_thread(const RVal (&x)[8]) {
    return red2<KIND>(red2<KIND>(red2<KIND>(x[0], x[1]), red2<KIND>(x[2], x[3])),
                      red2<KIND>(red2<KIND>(x[4], x[5]), red2<KIND>(x[6], x[7])));
}
// Butterfly over the warp: every lane ends with the same value (each step
// combines a commutative pair).
template <int KIND>
__device__ __forceinline__ RVal red_warp(RVal v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        RVal o;
        o.v = __shfl_xor_sync(0xffffffffu, v.v, m);
        o.i = KIND == RED_ARGMAX ? __shfl_xor_sync(0xffffffffu, v.i, m) : 0;
        v = red2<KIND>(v, o);
    }
    return v;
}
// The eight warps of a block, as ((w0 w1)(w2 w3))((w4 w5)(w6 w7)).
template <int KIND>
__device__ __forceinline__ RVal red_block8(const float* wv, const int64_t* wi) {
    RVal w[8];
#pragma unroll
    for (int k = 0; k < 8; k++) w[k] = {wv[k], KIND == RED_ARGMAX ? wi[k] : 0};
    return red2<KIND>(red2<KIND>(red2<KIND>(w[0], w[1]), red2<KIND>(w[2], w[3])),
                      red2<KIND>(red2<KIND>(w[4], w[5]), red2<KIND>(w[6], w[7])));
}
static_assert(kThreads == 256 && kG == 2, "the reduction tree assumes 8 warps of 2 x float4");

// A chunk's warp partials: A holds the values at positions
// cb + 4 (t + 256 k) + j; positions >= n take the identity. The chunk is
// G/2 blocks of the reduction tree (2048 positions, groups 2 sb and 2 sb + 1
// of block sb), the first being block blk0 of the launch; block b's warp w
// writes out[8 b + w] (and out_i), for the nblk blocks the launch has.
// ARGMAX inside one 2048-block: the index travels as a 32-bit offset in
// the block (the same order as the global index; INT32_MAX for "no
// element") and is widened once per warp partial.
struct RV32 {
    float v;
    int32_t o;
};
__device__ __forceinline__ RV32 am_pick32(const RV32& a, const RV32& b) {
    const bool na = a.v != a.v, nb = b.v != b.v;
    if (na || nb) return (na && nb ? a.o < b.o : na) ? a : b;
    if (a.v > b.v) return a;
    if (b.v > a.v) return b;
    const bool sa = __float_as_uint(a.v) >> 31, sb = __float_as_uint(b.v) >> 31;
    if (sa != sb) return sa ? b : a;
    return a.o < b.o ? a : b;
}
__device__ __forceinline__ RV32 am_warp32(const RV32 (&x)[8]) {
    RV32 v = am_pick32(am_pick32(am_pick32(x[0], x[1]), am_pick32(x[2], x[3])),
                       am_pick32(am_pick32(x[4], x[5]), am_pick32(x[6], x[7])));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        RV32 o;
        o.v = __shfl_xor_sync(0xffffffffu, v.v, m);
        o.o = __shfl_xor_sync(0xffffffffu, v.o, m);
        v = am_pick32(v, o);
    }
    return v;
}

template <int KIND, int G>
__device__ __forceinline__ void chunk_warps(const float4 (&A)[G], int64_t cb, int64_t n,
                                            int64_t idx_base, float* out, int64_t* out_i,
                                            int64_t blk0, int64_t nblk) {
    const int t = threadIdx.x;
#pragma unroll
    for (int sb = 0; sb < G / 2; sb++) {
        const int64_t b = blk0 + sb;
        if (b < nblk) {  // uniform over the block
            const int64_t base = cb + (int64_t)kChunk * sb;
            const bool full = base + kChunk <= n;
            if constexpr (KIND == RED_ARGMAX) {
                RV32 x[8];
#pragma unroll
                for (int k = 0; k < 2; k++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int32_t o = 4 * (t + kThreads * k) + e;
                        x[4 * k + e] = (full || base + o < n)
                                           ? RV32{f4_get(A[2 * sb + k], e), o}
                                           : RV32{__int_as_float((int)0xff800000u), INT32_MAX};
                    }
                const RV32 w = am_warp32(x);
                if ((t & 31) == 0) {
                    out[8 * b + (t >> 5)] = w.v;
                    out_i[8 * b + (t >> 5)] = w.o == INT32_MAX ? kNoIndex : idx_base + base + w.o;
                }
            } else {
                RVal x[8];
#pragma unroll
                for (int k = 0; k < 2; k++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int64_t p = base + 4 * (t + kThreads * k) + e;
                        x[4 * k + e] = (full || p < n) ? RVal{f4_get(A[2 * sb + k], e), 0}
                                                       : red_identity<KIND>();
                    }
                const RVal w = red_warp<KIND>(red_thread<KIND>(x));
                if ((t & 31) == 0) out[8 * b + (t >> 5)] = w.v;
            }
        }
    }
}
// Partial e of a level: entry e itself, or (warps8, the first level) the
// eight warp partials of chunk e combined.
template <int KIND>
__device__ __forceinline__ RVal red_entry(const float* v, const int64_t* vi, int64_t e,
                                          bool warps8) {
    if (warps8) return red_block8<KIND>(v + 8 * e, KIND == RED_ARGMAX ? vi + 8 * e : nullptr);
    return {v[e], KIND == RED_ARGMAX ? vi[e] : 0};
}

// One level of the reduction tree over m partials (value, index): block b
// reduces partials [kChunk b, kChunk b + kChunk) with the tree above into
// ov[b] (and oi[b]). With m = 0 one block writes the identity; with m = 1
// the partial is the result itself. `last`: the caller's result
// (red_final).
template <int KIND>
__global__ void __launch_bounds__(kThreads) k_red_level(const float* __restrict__ v,
                                                        const int64_t* __restrict__ vi, int64_t m,
                                                        float* ov, int64_t* oi, bool last,
                                                        bool warps8) {
    __shared__ float wv[8];
    __shared__ int64_t wi[8];
    const int t = threadIdx.x;
    if (m == 1) {  // no identity is added to a lone partial
        if (blockIdx.x == 0 && t == 0) {
            RVal b = red_entry<KIND>(v, vi, 0, warps8);
            if (last) b = red_final<KIND>(b);
            ov[0] = b.v;
            if (KIND == RED_ARGMAX) oi[0] = b.i;
        }
        return;
    }
    const int64_t base = (int64_t)blockIdx.x * kChunk;
    RVal x[8];
#pragma unroll
    for (int k = 0; k < kG; k++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t e = base + 4 * (t + kThreads * k) + j;
            x[4 * k + j] = e < m ? red_entry<KIND>(v, vi, e, warps8) : red_identity<KIND>();
        }
    const RVal r = red_warp<KIND>(red_thread<KIND>(x));
    if ((t & 31) == 0) {
        wv[t >> 5] = r.v;
        wi[t >> 5] = r.i;
    }
    __syncthreads();
    if (t == 0) {
        RVal b = red_block8<KIND>(wv, wi);
        if (last) b = red_final<KIND>(b);
        ov[blockIdx.x] = b.v;
        if (KIND == RED_ARGMAX) oi[blockIdx.x] = b.i;
    }
}

// Partials [from, to) set to the identity (a rank's slots past its own
// chunks in the sharded reduction's all-gather).
template <int KIND>
__global__ void k_red_fill(float* v, int64_t* vi, int64_t from, int64_t to) {
    const RVal id = red_identity<KIND>();
    for (int64_t e = from + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < to;
         e += (int64_t)gridDim.x * blockDim.x) {
        v[e] = id.v;
        if (vi) vi[e] = id.i;
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

// The input span a chunk needs: with its halo (the first chunk of a block's
// range, whose window heads are computed) or without (later chunks carry
// the heads over from the chunk before).
__device__ __forceinline__ ChunkSpan chunk_span(int64_t cb, int hs, int64_t n, int64_t halo,
                                                bool with_halo, int chunk) {
    ChunkSpan s;
    s.org = cb - hs;
    s.lo = max(with_halo ? s.org : cb, -halo);
    s.hi = min(cb + (int64_t)chunk, n);
    s.len4 = s.hi > s.lo ? ((s.hi - s.lo) & ~int64_t(3)) : 0;
    return s;
}

// Shared memory (float4 units): meta | taps (n_fir x kMaxTaps floats) |
// tiles (tile_floats(head) floats each) | temporaries (n_tmp x kChunk floats) |
// stages (nst x n_in x (hs + kChunk) floats, BULK only). Input k of a stage
// holds positions [cb - hs, cb + kChunk) of the chunk at cb (the part below
// cb only for the first chunk of the block's range).
//
// A block works through a contiguous range of chunks. Window f's tile holds
// positions [cb - head, cb + kChunk): the chunk's own positions are staged
// by one run of the window's program; the head below cb is the previous
// chunk's last head positions, copied within the tile, and is computed by
// a short head run only for the first chunk of the range. head is the
// window's reach (window_reach(taps)), plus, when later windows read it
// (chained windows), the largest head among them: their head runs read it
// that far below the chunk.
//
// Bulk-copy mode (BULK): the chunk's inputs travel HBM -> shared memory by
// cp.async.bulk, one copy per input, in `nst` stages that complete on
// per-stage mbarriers, so nst-1 chunks stream in while one is interpreted.
// Requires every input 16-byte aligned and halo = 0 mod 4. Otherwise
// (DIRECT) the interpreter reads input operands from HBM itself.
//
// A reduction (P.reduce) writes no output array: each warp's values of
// chunk c (its index in the launch) are reduced (red_thread, red_warp) into
// out[8 c + warp] and, for ARGMAX, out_idx[8 c + warp]; idx_base + p is the
// index of position p. The level kernels combine the eight warps.
//
// A graph without windows has no shared value that one thread writes and
// another reads (temporaries and staged operands are per thread): its warps
// run ahead of each other, and the last of the eight warps to finish with a
// stage (a shared counter per stage) refills it, instead of thread 0 after a
// block barrier.
template <bool BULK, int G>
__global__ void __launch_bounds__(kThreads, G == kG ? 3 : 2)
    k_tile(const __grid_constant__ Program P, float* __restrict__ out, int64_t n, int64_t halo,
           bool vec, bool in_vec, int32_t hs, int32_t stages4, int32_t nst, uint32_t* wd,
           int64_t* __restrict__ out_idx, int64_t idx_base) {
    constexpr int CH = chunk_of(G), CH4 = CH / 4;
    __shared__ __align__(8) uint64_t bars[kMaxStages];   // stage s loaded
    __shared__ int rel[kMaxStages];  // warps done with stage s (window-free graphs)
    extern __shared__ float4 sm4[];
    const int code_cap = meta_code_cap(P.n_code);
    Insn* code_s = reinterpret_cast<Insn*>(sm4);
    int4* fir_s = reinterpret_cast<int4*>(code_s + code_cap);
    const float** in_s = reinterpret_cast<const float**>(fir_s + P.n_fir);
    float* taps_s = reinterpret_cast<float*>(sm4) + meta_bytes(P.n_code, P.n_in, P.n_fir) / 4;
    const int32_t sstride = hs + CH;  // floats per staged input
    const int32_t stage_floats = P.n_in * sstride;
    float* stages = reinterpret_cast<float*>(sm4 + stages4);
    const int tid = threadIdx.x;
    const int64_t nchunks = (n + CH - 1) / CH;
    for (int i = tid; i < code_cap; i += kThreads)
        code_s[i] = i < P.n_code ? P.code[i] : Insn{OP_END, F_END, 0, 0, 0, 0.0f, 0};
    for (int k = tid; k < P.n_in; k += kThreads) in_s[k] = P.in[k];
    for (int f = tid; f < P.n_fir; f += kThreads)
        fir_s[f] = make_int4(P.fir[f].start, P.fir[f].taps, P.fir[f].head, P.fir[f].tile4);
    for (int f = 0; f < P.n_fir; f++)
        for (int k = tid; k < kMaxTaps; k += kThreads)
            taps_s[f * kMaxTaps + k] = P.fir[f].h[k];  // zero past taps

    const int64_t per_block = (nchunks + gridDim.x - 1) / gridDim.x;
    const int64_t c0 = blockIdx.x * per_block;
    const int64_t c1 = min(c0 + per_block, nchunks);
    auto issue = [&](int64_t c, int s) {
        const ChunkSpan sp = chunk_span(c * CH, hs, n, halo, c == c0, CH);
        mbar_arrive_expect_tx(&bars[s], (uint32_t)(sp.len4 * 4 * P.n_in));
        if (sp.len4 > 0)
            for (int k = 0; k < P.n_in; k++)
                bulk_g2s(stages + s * stage_floats + k * sstride + (sp.lo - sp.org),
                         in_s[k] + sp.lo, (uint32_t)(sp.len4 * 4), &bars[s]);
    };
    if (BULK) {
        if (tid == 0) {
            for (int s = 0; s < nst; s++) {
                mbar_init(&bars[s], 1);
                rel[s] = 0;
            }
            fence_mbar_init();
        }
        __syncthreads();
        if (tid == 0)
            for (int s = 0; s < nst; s++)
                if (c0 + s < c1) issue(c0 + s, s);
    }
    __syncthreads();

    Ctx cx;
    cx.S = sm4;
    cx.taps_s = taps_s;
    cx.fir = fir_s;
    cx.in = in_s;
    cx.out = out;
    cx.n = n;
    cx.halo = halo;
    cx.vec = vec;
    cx.in_vec = in_vec;
    const int nf = P.n_fir;
    const bool free_run = nf == 0;
    float4 A[G];  // the last run's values (the main program's, for a reduction)
    int it = 0;
    for (int64_t c = c0; c < c1; c++, it++) {
        const int64_t cb = c * CH;
        const bool first = c == c0;
        const ChunkSpan sp = chunk_span(cb, hs, n, halo, first, CH);
        int s = 0;
        if (BULK) {
            s = it % nst;
            if (!mbar_wait(&bars[s], (uint32_t)((it / nst) & 1), wd)) {
                // Gave up (the watchdog is raised): let the block's other
                // copies in flight land, each wait bounded, before exiting.
                for (int j = 1; j < nst && c + j < c1; j++)
                    mbar_wait(&bars[(it + j) % nst], (uint32_t)(((it + j) / nst) & 1), wd);
                return;
            }
            float* buf = stages + s * stage_floats;
            // The last 0-3 samples of a ragged signal are not a whole 16-byte
            // unit: plain loads.
            const int64_t tail = sp.hi - (sp.lo + sp.len4);
            if (tail > 0) {  // uniform over the block
                if (tid < P.n_in * 4) {
                    const int k = tid / 4, e = tid % 4;
                    const int64_t pos = sp.lo + sp.len4 + e;
                    if (e < tail) buf[k * sstride + (pos - sp.org)] = in_s[k][pos];
                }
                __syncthreads();
            }
        }
        const int32_t in4 = stages4 + s * stage_floats / 4;
        const bool edge = cb - (int64_t)hs < -halo || cb + CH > n;
        // Jobs 2f and 2f+1 stage window f: its head (first chunk only) and
        // the chunk itself; job 2 nf is the main program over the chunk. One
        // loop, so the interpreter is inlined once per form.
        for (int j = 0; j <= 2 * nf; j++) {
            Run r;
            int pc;
            if (j < 2 * nf) {
                const int4 fd = fir_s[j >> 1];
                const int head4 = fd.z / 4;
                pc = fd.x;
                if (!(j & 1)) {  // head: tile [0, head) = positions [cb - head, cb)
                    r.sh_in = in4 + (hs - fd.z) / 4;
                    r.sh_st = 0;
                    r.woff4 = -head4;
                    r.gm = first && tid < head4 ? 1u : 0u;
                    r.p0 = cb - fd.z;
                } else {  // the chunk: tile [head, head + CH)
                    // Carry the head over: the previous chunk's last head
                    // positions sit at tile [CH, CH + head). The
                    // thread that copies a float4 is the one whose staging
                    // below overwrites it, so no barrier is needed.
                    if (!first && tid >= kThreads - head4) {
                        float4* tile = cx.S + fd.w;
                        const int q = tid - (kThreads - head4);
                        tile[q] = tile[CH4 + q];
                    }
                    r.sh_in = in4 + hs / 4;
                    r.sh_st = head4;
                    r.woff4 = 0;
                    r.gm = (1u << G) - 1;
                    r.p0 = cb;
                }
            } else {
                pc = P.main_start;
                r.sh_in = in4 + hs / 4;
                r.sh_st = 0;
                r.woff4 = 0;
                r.gm = (1u << G) - 1;
                r.p0 = cb;
            }
            r.edge = edge;
            if (r.gm == (1u << G) - 1)
                interpret<BULK, true, G>(code_s, pc, cx, r, A);
            else if (r.gm)
                interpret<BULK, false, G>(code_s, pc, cx, r, A);
            // Windows staged before the main program reads them, and a
            // window before a later window's staging reads it (chains).
            if ((j & 1) && (j + 1 == 2 * nf || (fir_s[j >> 1].y & kSyncAfter))) __syncthreads();
        }
        if (P.reduce != RED_NONE) {
            const int64_t b0 = c * (G / 2), nb = (n + kChunk - 1) / kChunk;
            float* o = out;
            int64_t* oi = out_idx;
            switch (P.reduce) {  // uniform: one branch per chunk
                case RED_SUM: chunk_warps<RED_SUM, G>(A, cb, n, idx_base, o, oi, b0, nb); break;
                case RED_MIN: chunk_warps<RED_MIN, G>(A, cb, n, idx_base, o, oi, b0, nb); break;
                case RED_MAX: chunk_warps<RED_MAX, G>(A, cb, n, idx_base, o, oi, b0, nb); break;
                default: chunk_warps<RED_ARGMAX, G>(A, cb, n, idx_base, o, oi, b0, nb); break;
            }
        }
        if (BULK) {
            // Every thread is done with this stage (and, with windows, with
            // the tiles and temporaries); order its generic accesses before
            // the next bulk copy into it.
            fence_proxy_async_smem();
            if (free_run) {
                // The counter's read-modify-writes, fenced on both sides, order
                // every warp's reads of the stage before the refill. The reset
                // precedes the refill's arrive (a release), which every warp
                // acquires before it counts this stage again.
                __syncwarp();
                if ((tid & 31) == 0) {
                    __threadfence_block();
                    if (atomicAdd(&rel[s], 1) == kThreads / 32 - 1) {
                        __threadfence_block();
                        rel[s] = 0;
                        if (c + nst < c1) issue(c + nst, s);
                    }
                }
            } else {
                __syncthreads();
                if (tid == 0 && c + nst < c1) issue(c + nst, s);
            }
        } else if (!free_run) {
            __syncthreads();  // the tiles are rewritten by the next chunk
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
    bool chained = false;  // FIR of an expression with a FIR accepted (opt-in)
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

// Whether the expression at id reads window node w directly (not through
// another window).
bool reads_window(const simtgo_tile_graph* g, int id, int w) {
    if (id == w) return true;
    const Node& n = g->nodes[id];
    if (n.kind == K_FIR) return false;
    return (n.a >= 0 && reads_window(g, n.a, w)) || (n.b >= 0 && reads_window(g, n.b, w));
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

// A lowered instruction, before the shared-memory layout of a launch gives
// its operand an address.
enum Space : uint8_t { SP_NONE = 0, SP_IN, SP_TMP, SP_WIN, SP_SELF };
struct LInsn {
    uint8_t op;
    uint8_t space;
    uint16_t idx;  // input, temporary or window index
    float imm;
};

// A device instruction before the layout gives its operands addresses: a
// fused run of lowered steps (see tilek::Insn).
struct FInsn {
    uint8_t op = tilek::OP_END;  // the operation, or OP_END for none
    bool loada = false, sta = false, stage = false, store = false, end = false;
    uint8_t a_space = SP_NONE, b_space = SP_NONE;
    uint16_t a_idx = 0, b_idx = 0;  // b: binary operand, or the FIRACC window
    uint16_t d_idx = 0;             // the STA temporary or the STAGE window
    float imm = 0.0f;
};

// Fuses a program's steps into device instructions: each takes an optional
// load, one operation, an optional store to a temporary, to a window tile or
// to the output, and the end, in that order.
void fuse(const std::vector<LInsn>& raw, std::vector<FInsn>& out) {
    FInsn cur;
    bool open = false;
    auto flush = [&]() {
        if (open) out.push_back(cur);
        cur = FInsn();
        open = false;
    };
    for (const LInsn& li : raw) {
        switch (li.op) {
            case tilek::OP_LDA:
                flush();
                cur.loada = true;
                cur.a_space = li.space;
                cur.a_idx = li.idx;
                open = true;
                break;
            case tilek::OP_STA:
                if (!open || cur.sta || cur.stage || cur.store) flush();
                cur.sta = true;
                cur.d_idx = li.idx;
                open = true;
                break;
            case tilek::OP_STAGE:
            case tilek::OP_STORE:
                if (!open || cur.stage || cur.store) flush();
                if (li.op == tilek::OP_STAGE) {
                    if (cur.sta) flush();
                    cur.stage = true;
                    cur.d_idx = li.idx;
                } else {
                    cur.store = true;
                }
                open = true;
                break;
            case tilek::OP_END:
                cur.end = true;
                open = true;
                flush();
                break;
            default:  // an operation: joins a pending load, else starts anew
                if (open && !(cur.op == tilek::OP_END && !cur.sta && !cur.stage && !cur.store))
                    flush();
                cur.op = li.op;
                cur.b_space = li.space;
                cur.b_idx = li.idx;
                cur.imm = li.imm;
                open = true;
        }
    }
    flush();
}

struct Lowered {
    std::vector<FInsn> code;
    int32_t main_start = 0;
    std::vector<int32_t> fir_start;  // pc of each window's staging program
    int n_tmp = 0;                   // temporaries the programs use at once
    std::vector<int> in_nodes;       // data input node ids, in input order
    std::vector<int> fir_nodes;      // window node ids, in window order
    std::vector<int> param_of;       // reference parameter index pK of each data input
    int32_t reduce = tilek::RED_NONE;  // the main program's value is reduced, not stored
    std::vector<int32_t> head;       // each window's head (positions below the chunk)
    std::vector<char> sync_after;    // a later window's staging reads this window
};

// Emits one program for the accumulator machine: a window's signal (ending
// in STAGE) or the main program (ending in STORE). Values live in the
// accumulator; a value with uses still to come is stored once to a
// temporary. A binary node whose operands are both unstored evaluates the
// operand that needs more temporaries first, stores it, then the other
// (Sethi-Ullman order). In the main program a window node is FIRACC, and a
// window's signal root is read from the window's tile rather than computed
// again.
struct Gen {
    const simtgo_tile_graph* g;
    bool main;
    Lowered& L;
    std::unordered_map<int, int>& input_index;
    const std::unordered_map<int, int>& fir_index;
    std::vector<int> uses;         // references still to be consumed, per node
    std::vector<int8_t> space;     // where a node's value is stored (Space), or SP_NONE
    std::vector<int> where;        // its index in that space
    std::vector<int> need_memo;
    std::vector<LInsn> raw;        // the program's steps, fused at the end
    bool tmp_busy[tilek::kMaxTmp] = {};
    int status = 0;                // -1 temporaries exhausted, -2 inputs exhausted

    Gen(const simtgo_tile_graph* g_, bool main_, Lowered& L_, std::unordered_map<int, int>& ii,
        const std::unordered_map<int, int>& fi)
        : g(g_), main(main_), L(L_), input_index(ii), fir_index(fi) {
        const size_t nn = g->nodes.size();
        uses.assign(nn, 0);
        space.assign(nn, SP_NONE);
        where.assign(nn, -1);
        need_memo.assign(nn, -1);
    }
    void push(uint8_t op, uint8_t sp = SP_NONE, int idx = 0, float imm = 0.0f) {
        raw.push_back(LInsn{op, sp, (uint16_t)idx, imm});
    }
    // A window node is a leaf of every program that reads it (FIRACC of its
    // staged tile): the main program, and with chained windows a later
    // window's staging.
    bool leaf(int id) const {
        const Node& n = g->nodes[id];
        return n.kind == K_INPUT || n.kind == K_FIR;
    }
    // Counts references inside this program.
    void count(int root) {
        std::vector<int> order;
        std::vector<char> seen(g->nodes.size(), 0);
        postorder(g, root, order, seen, true);
        for (int id : order) {
            if (leaf(id)) continue;
            const Node& n = g->nodes[id];
            if (n.a >= 0) uses[n.a]++;
            if (n.b >= 0) uses[n.b]++;
        }
    }
    // Temporaries an unstored node needs while it is evaluated.
    int need(int id) {
        if (space[id] != SP_NONE || leaf(id)) return 0;
        if (need_memo[id] >= 0) return need_memo[id];
        const Node& n = g->nodes[id];
        int r;
        if (n.b < 0 || n.a == n.b) {
            r = need(n.a);
        } else if (space[n.a] != SP_NONE || leaf(n.a) || space[n.b] != SP_NONE || leaf(n.b)) {
            r = std::max(need(n.a), need(n.b));
        } else {
            const int na = need(n.a), nb = need(n.b);
            r = na == nb ? na + 1 : std::max(na, nb);
        }
        return need_memo[id] = r;
    }
    int alloc_tmp() {
        for (int j = 0; j < tilek::kMaxTmp; j++)
            if (!tmp_busy[j]) {
                tmp_busy[j] = true;
                L.n_tmp = std::max(L.n_tmp, j + 1);
                return j;
            }
        status = -1;
        return -1;
    }
    void consume(int id) {
        if (--uses[id] == 0 && space[id] == SP_TMP) {
            tmp_busy[where[id]] = false;
            space[id] = SP_NONE;
        }
    }
    // The memory operand of a stored node or an input, or false.
    bool operand(int id, uint8_t* sp, int* idx) {
        const Node& n = g->nodes[id];
        if (space[id] != SP_NONE) {
            *sp = (uint8_t)space[id];
            *idx = where[id];
            return true;
        }
        if (n.kind == K_INPUT) {
            auto it = input_index.find(id);
            int k;
            if (it == input_index.end()) {
                k = (int)L.in_nodes.size();
                if (k >= tilek::kMaxIn) {
                    status = -2;
                    return false;
                }
                input_index[id] = k;
                L.in_nodes.push_back(id);
            } else {
                k = it->second;
            }
            *sp = SP_IN;
            *idx = k;
            return true;
        }
        return false;
    }
    bool stored(int id) { return space[id] != SP_NONE || g->nodes[id].kind == K_INPUT; }
    // Leaves the value of id in the accumulator.
    void emit(int id) {
        if (status) return;
        uint8_t sp;
        int idx;
        if (operand(id, &sp, &idx)) {
            push(tilek::OP_LDA, sp, idx);
            return;
        }
        if (status) return;
        const Node& n = g->nodes[id];
        if (n.kind == K_FIR) {
            push(tilek::OP_FIRACC, SP_NONE, fir_index.at(id));
        } else if (n.kind == K_SCALE || n.kind == K_SQRT || n.kind == K_ABS) {
            emit(n.a);
            consume(n.a);
            if (n.kind == K_SCALE) push(tilek::OP_SCALE, SP_NONE, 0, n.scale);
            if (n.kind == K_SQRT) push(tilek::OP_SQRT);
            if (n.kind == K_ABS) push(tilek::OP_ABS);
        } else {
            const uint8_t op = n.kind == K_ADD   ? tilek::OP_ADD
                               : n.kind == K_MUL ? tilek::OP_MUL
                                                 : tilek::OP_HYPOT;
            if (n.a == n.b) {
                emit(n.a);
                consume(n.a);
                consume(n.a);
                push(op, SP_SELF);
            } else {
                // The operand kept in memory: one already stored, else the
                // one evaluated first (and stored) -- the needier one.
                int first = n.b, second = n.a;
                if (stored(n.a) && !stored(n.b)) {
                    first = n.a;
                    second = n.b;
                } else if (!stored(n.b) && need(n.a) > need(n.b)) {
                    first = n.a;
                    second = n.b;
                }
                if (!stored(first)) {
                    emit(first);
                    if (status) return;
                    if (space[first] == SP_NONE) {  // not stored by emit: keep it for this use
                        const int j = alloc_tmp();
                        if (j < 0) return;
                        push(tilek::OP_STA, SP_TMP, j);
                        space[first] = SP_TMP;
                        where[first] = j;
                    }
                }
                emit(second);
                if (status) return;
                if (!operand(first, &sp, &idx)) {
                    status = status ? status : -1;
                    return;
                }
                push(op, sp, idx);
                consume(second);
                consume(first);
            }
        }
        if (status) return;
        // More uses to come after the current one: store it once.
        if (uses[id] > 1 && space[id] == SP_NONE) {
            const int j = alloc_tmp();
            if (j < 0) return;
            push(tilek::OP_STA, SP_TMP, j);
            space[id] = SP_TMP;
            where[id] = j;
        }
    }
};

// Lowers the graph rooted at root (its value reduced by `reduce` instead of
// stored, unless RED_NONE). Returns 0 or a status (message recorded).
int lower(const simtgo_tile_graph* g, int root, Lowered& L, int32_t reduce = tilek::RED_NONE) {
    L = Lowered();
    L.reduce = reduce;
    // The reference's parameter numbering: every input node, taps included,
    // in postorder (tile/codegen.go:24-35).
    {
        std::vector<int> order;
        std::vector<char> seen(g->nodes.size(), 0);
        postorder(g, root, order, seen, false);
        int p = 0;
        L.param_of.assign(g->nodes.size(), -1);
        for (int id : order)
            if (g->nodes[id].kind == K_INPUT) L.param_of[id] = p++;
        for (int id : order)
            if (g->nodes[id].kind == K_FIR) L.fir_nodes.push_back(id);
    }
    if ((int)L.fir_nodes.size() > tilek::kMaxFir)
        return sg::fail(SIMTGO_ESIZE, "tile: %zu windowed operations; the fused kernel stages at most %d",
                        L.fir_nodes.size(), tilek::kMaxFir);
    std::unordered_map<int, int> fir_index, input_index;
    const int nfw = (int)L.fir_nodes.size();
    for (int i = 0; i < nfw; i++) fir_index[L.fir_nodes[i]] = i;
    // Heads: a window read by later windows' staging (chained windows; the
    // windows are in postorder, so readers come later) reaches below the
    // chunk by its own reach plus the largest head among its readers.
    L.head.assign(nfw, 0);
    L.sync_after.assign(nfw, 0);
    for (int i = nfw - 1; i >= 0; i--) {
        const int taps = (int)g->nodes[g->nodes[L.fir_nodes[i]].b].taps.size();
        int below = 0;
        for (int j = i + 1; j < nfw; j++)
            if (reads_window(g, g->nodes[L.fir_nodes[j]].a, L.fir_nodes[i])) {
                below = std::max(below, L.head[j]);
                L.sync_after[i] = 1;
            }
        L.head[i] = tilek::window_reach(taps) + below;
    }
    if (nfw > 0 && *std::max_element(L.head.begin(), L.head.end()) > 4 * tilek::kThreads)
        return sg::fail(SIMTGO_ESIZE, "tile: chained windows reach more than %d samples below a chunk",
                        4 * tilek::kThreads);
    int status = 0;
    for (size_t f = 0; f < L.fir_nodes.size() && !status; f++) {
        const int sig = g->nodes[L.fir_nodes[f]].a;
        L.fir_start.push_back((int32_t)L.code.size());
        Gen gen(g, false, L, input_index, fir_index);
        gen.count(sig);
        gen.uses[sig]++;  // the STAGE
        gen.emit(sig);
        gen.push(tilek::OP_STAGE, SP_NONE, (int)f);
        gen.push(tilek::OP_END);
        fuse(gen.raw, L.code);
        status = gen.status;
    }
    if (!status) {
        L.main_start = (int32_t)L.code.size();
        Gen gen(g, true, L, input_index, fir_index);
        gen.count(root);
        gen.uses[root]++;  // the STORE
        // Each window's signal root is in its tile over the chunk.
        for (size_t f = 0; f < L.fir_nodes.size(); f++) {
            const int sig = g->nodes[L.fir_nodes[f]].a;
            if (g->nodes[sig].kind != K_INPUT && gen.space[sig] == SP_NONE) {
                gen.space[sig] = SP_WIN;
                gen.where[sig] = (int)f;
            }
        }
        gen.emit(root);
        if (reduce == tilek::RED_NONE) gen.push(tilek::OP_STORE);
        gen.push(tilek::OP_END);
        fuse(gen.raw, L.code);
        status = gen.status;
    }
    if (status == -2)
        return sg::fail(SIMTGO_ESIZE, "tile: more than %d distinct inputs", tilek::kMaxIn);
    if (status == -1)
        return sg::fail(SIMTGO_ESIZE,
                        "tile: the graph keeps more than %d values live at once; materialise part of it",
                        tilek::kMaxTmp);
    if (L.code.size() > (size_t)tilek::kMaxCode)
        return sg::fail(SIMTGO_ESIZE, "tile: the program has %zu instructions (max %d)",
                        L.code.size(), tilek::kMaxCode);
    return 0;
}

// Float4 offset of window f's tile among the tiles.
int32_t tile_off4(const Lowered& L, int f) {
    int32_t off = 0;
    for (int i = 0; i < f; i++) off += tilek::tile_floats(L.head[i]) / 4;
    return off;
}

// The launch's shared-memory layout (float4 offsets) and its program.
struct Layout {
    int32_t taps4, tiles4, temps4, stages4, sstride, nst;
    int32_t g;  // float4 groups per thread (the interpreter's G); chunk = 1024 g
    size_t smem;
};

void build_program(const simtgo_tile_graph* g, const Lowered& L, const Layout& Y, bool bulk,
                   tilek::Program& P) {
    memset(&P, 0, sizeof P);
    P.main_start = L.main_start;
    P.reduce = L.reduce;
    P.n_fir = (int32_t)L.fir_nodes.size();
    P.n_in = (int32_t)L.in_nodes.size();
    P.n_code = (int32_t)L.code.size();
    for (int f = 0; f < P.n_fir; f++) {
        const Node& fn = g->nodes[L.fir_nodes[f]];
        const std::vector<float>& h = g->nodes[fn.b].taps;
        P.fir[f].start = L.fir_start[f];
        P.fir[f].taps = (int32_t)h.size() | (L.sync_after[f] ? tilek::kSyncAfter : 0);
        P.fir[f].head = L.head[f];
        P.fir[f].tile4 = Y.tiles4 + tile_off4(L, f);
        for (size_t k = 0; k < h.size(); k++) P.fir[f].h[k] = h[k];
    }
    // A lowered operand's address: inputs relative to the run's stage
    // (BULK) or their index (DIRECT), temporaries and window signals absolute.
    auto addr = [&](uint8_t space, int idx, bool* input) -> uint16_t {
        *input = space == SP_IN;
        switch (space) {
            case SP_IN: return (uint16_t)(bulk ? idx * Y.sstride / 4 : idx);
            case SP_TMP: return (uint16_t)(Y.temps4 + idx * tilek::chunk_of(Y.g) / 4);
            case SP_WIN: return (uint16_t)(P.fir[idx].tile4 + P.fir[idx].head / 4);
            default: return (uint16_t)idx;
        }
    };
    for (size_t pc = 0; pc < L.code.size(); pc++) {
        const FInsn& fi = L.code[pc];
        tilek::Insn& in = P.code[pc];
        memset(&in, 0, sizeof in);
        in.op = fi.op;
        in.imm = fi.imm;
        bool input;
        if (fi.loada) {
            in.flags |= tilek::F_LOADA;
            in.a = addr(fi.a_space, fi.a_idx, &input);
            if (input) in.flags |= tilek::F_IN_A;
        }
        if (fi.op == tilek::OP_FIRACC) {
            in.b = fi.b_idx;
        } else if (fi.b_space == SP_SELF) {
            in.flags |= tilek::F_SELF;
        } else if (fi.b_space != SP_NONE) {
            in.b = addr(fi.b_space, fi.b_idx, &input);
            if (input) in.flags |= tilek::F_IN_B;
        }
        if (fi.sta) {
            in.flags |= tilek::F_STA;
            in.d = (uint16_t)(Y.temps4 + fi.d_idx * tilek::chunk_of(Y.g) / 4);
        }
        if (fi.stage) {
            in.flags |= tilek::F_STAGE;
            in.d = fi.d_idx;
        }
        if (fi.store) in.flags |= tilek::F_STORE;
        if (fi.end) in.flags |= tilek::F_END;
    }
}

// Launches a lowered program. dev_in[k] = device data of L.in_nodes[k] (halo
// elements first).
// For a reduction, out (and out_idx, ARGMAX) receive eight warp partials per
// 2048-element block and idx_base is the index of element 0.
int launch_program(const simtgo_tile_graph* g, const Lowered& L,
                   const std::vector<const float*>& dev_in, float* out, int64_t n, int64_t halo,
                   cudaStream_t s, int64_t* out_idx = nullptr, int64_t idx_base = 0) {
    const sg::DevInfo* d;
    int rc;
    if ((rc = sg::current_device(&d))) return rc;
    if (n <= 0) return 0;
    const int n_in = (int)L.in_nodes.size(), n_fir = (int)L.fir_nodes.size();
    bool in_aligned = true;
    for (const float* p : dev_in) in_aligned = in_aligned && sg::aligned16(p);
    const bool vec = sg::aligned16(out);
    // Samples a chunk's windows reach below it.
    int32_t hs = 0;
    for (int f = 0; f < n_fir; f++) hs = std::max<int32_t>(hs, L.head[f]);
    Layout Y;
    // Four groups per thread for graphs without windows or Hypot.
    bool hypot = false;
    for (const FInsn& fi : L.code) hypot = hypot || fi.op == tilek::OP_HYPOT;
    Y.g = n_fir == 0 && !hypot ? tilek::kGWide : tilek::kG;
    const int chunk = tilek::chunk_of(Y.g);
    Y.taps4 = tilek::meta_bytes((int)L.code.size(), n_in, n_fir) / 16;
    Y.tiles4 = Y.taps4 + n_fir * tilek::kMaxTaps / 4;
    Y.temps4 = Y.tiles4 + tile_off4(L, n_fir);
    Y.stages4 = Y.temps4 + L.n_tmp * chunk / 4;
    Y.sstride = hs + chunk;
    const size_t base_smem = (size_t)Y.stages4 * 16;
    const size_t stage_bytes = (size_t)n_in * Y.sstride * sizeof(float);
    // Every instantiation may take up to the opt-in maximum of dynamic
    // shared memory (less 1 KB for the static mbarriers).
    const int dyn_max = d->max_smem_optin - 1024;
    static std::atomic<uint64_t> configured{0};
    const uint64_t dev_bit = 1ull << (d->device & 63);
    using tilek::kG;
    using tilek::kGWide;
    if (!(configured.load() & dev_bit)) {
        for (auto k : {tilek::k_tile<true, kG>, tilek::k_tile<false, kG>,
                       tilek::k_tile<true, kGWide>, tilek::k_tile<false, kGWide>}) {
            rc = sg::cuda_status(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      dyn_max),
                                 "cudaFuncSetAttribute(tile)");
            if (rc) return rc;
        }
        configured.fetch_or(dev_bit);
    }
    // Blocks per SM and input stages: registers bound the blocks; each
    // block's stages take its share of the SM's shared memory. The choice is
    // the most blocks whose stages keep >= 64 KB per SM in flight (HBM
    // latency x bandwidth per SM), else the most bytes in flight. With
    // unaligned inputs, or fewer than two stages' room, the inputs are read
    // from HBM by the interpreter itself (DIRECT).
    int reg_blocks = 0;
    rc = sg::cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                             &reg_blocks,
                             Y.g == kG ? tilek::k_tile<true, kG> : tilek::k_tile<true, kGWide>,
                             tilek::kThreads, base_smem),
                         "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
    if (rc) return rc;
    bool bulk = false;
    Y.nst = 0;
    if (in_aligned && halo % 4 == 0 && n_in > 0) {
        int64_t best_inflight = -1;
        for (int per_sm = std::max(1, reg_blocks); per_sm >= 1; per_sm--) {
            const int64_t share =
                std::min<int64_t>(dyn_max, d->smem_per_sm / per_sm - 2048);
            const int64_t fit = (share - (int64_t)base_smem) / (int64_t)stage_bytes;
            const int nst = (int)std::min<int64_t>(fit, tilek::kMaxStages);
            if (nst < 2) continue;
            const int64_t inflight = (int64_t)per_sm * (nst - 1) * (int64_t)stage_bytes;
            if (inflight > best_inflight) {
                best_inflight = inflight;
                Y.nst = nst;
            }
            if (inflight >= 64 * 1024) {
                Y.nst = nst;
                break;
            }
        }
        bulk = Y.nst >= 2;
    }
    Y.smem = bulk ? base_smem + Y.nst * stage_bytes : base_smem;
    if (Y.smem > (size_t)dyn_max)
        return sg::fail(SIMTGO_ESIZE, "tile: the program needs %zu bytes of shared memory (max %d)",
                        Y.smem, dyn_max);
    static thread_local tilek::Program P;
    build_program(g, L, Y, bulk, P);
    for (int k = 0; k < n_in; k++) P.in[k] = dev_in[k];  // element 0; [-halo, 0) precede it
    auto kern = Y.g == kG ? (bulk ? tilek::k_tile<true, kG> : tilek::k_tile<false, kG>)
                          : (bulk ? tilek::k_tile<true, kGWide> : tilek::k_tile<false, kGWide>);
    int per_sm = 0;
    rc = sg::cuda_status(
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, tilek::kThreads, Y.smem),
        "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
    if (rc) return rc;
    // Whole waves of resident blocks, up to eight, each block over a
    // contiguous range of at least 32 chunks: a block that finishes early is
    // replaced by the next one, so SMs that see HBM faster take more of the
    // signal (measured 1-10% faster than one persistent wave on the two-die
    // B200 at 2^28 elements). Short signals keep one wave: every range starts
    // with a pipeline fill and, with windows, a head run, and a partial wave
    // would leave most SMs idle at the end.
    const int64_t chunks = sg::ceil_div(n, (int64_t)chunk);
    const int64_t resident = (int64_t)d->sms * std::max(1, per_sm);
    const int64_t waves = std::max<int64_t>(1, std::min<int64_t>(8, chunks / (32 * resident)));
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(chunks, waves * resident));
    sg::before_launch();
    kern<<<blocks, tilek::kThreads, Y.smem, s>>>(P, out, n, halo, vec, in_aligned, hs, Y.stages4,
                                                 Y.nst, sg::watchdog_device_ptr(), out_idx,
                                                 idx_base);
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
    return launch_program(g, L, dev_in, out, n, halo, s);
}

// ---- reductions ----------------------------------------------------------------

// Stream-ordered device scratch, released on its stream when it goes out of
// scope (after everything enqueued before).
struct AsyncBuf {
    void* p = nullptr;
    cudaStream_t s = 0;
    ~AsyncBuf() {
        if (p) cudaFreeAsync(p, s);
    }
    int alloc(size_t bytes, cudaStream_t st) {
        s = st;
        return sg::cuda_status(cudaMallocAsync(&p, std::max<size_t>(bytes, 16), st),
                               "cudaMallocAsync");
    }
};

int64_t n_partials(int64_t n) { return (n + tilek::kChunk - 1) / tilek::kChunk; }
// Entries the levels above m partials need (each level but the last).
int64_t upper_slots(int64_t m) {
    int64_t total = 0;
    while (m > tilek::kChunk) {
        m = n_partials(m);
        total += m;
    }
    return total + 1;
}

// Reduces m chunk partials (given as their warp partials: v, and vi for
// ARGMAX) into the caller's value (and index): one k_red_level launch per
// level of the tree; uv/ui hold the levels between.
int red_level(int kind, unsigned blocks, const float* v, const int64_t* vi, int64_t m, float* ov,
              int64_t* oi, bool last, bool w8, cudaStream_t s) {
    using namespace tilek;
    sg::before_launch();
    switch (kind) {
        case RED_SUM: k_red_level<RED_SUM><<<blocks, kThreads, 0, s>>>(v, vi, m, ov, oi, last, w8); break;
        case RED_MIN: k_red_level<RED_MIN><<<blocks, kThreads, 0, s>>>(v, vi, m, ov, oi, last, w8); break;
        case RED_MAX: k_red_level<RED_MAX><<<blocks, kThreads, 0, s>>>(v, vi, m, ov, oi, last, w8); break;
        default: k_red_level<RED_ARGMAX><<<blocks, kThreads, 0, s>>>(v, vi, m, ov, oi, last, w8);
    }
    return sg::launch_status("tile reduce");
}

// v/vi: the eight warp partials of each of m chunks (the interpreter's
// output), 8 m entries.
int finish_levels(int kind, const float* v, const int64_t* vi, int64_t m, float* value,
                  int64_t* index, cudaStream_t s, float* uv, int64_t* ui) {
    const bool am = kind == tilek::RED_ARGMAX;
    if (m <= 1) return red_level(kind, 1, v, vi, m, value, am ? index : nullptr, true, true, s);
    bool w8 = true;
    while (m > 1) {
        const int64_t nb = n_partials(m);
        const bool last = nb == 1;
        float* ov = last ? value : uv;
        int64_t* oi = am ? (last ? index : ui) : nullptr;
        if (int rc = red_level(kind, (unsigned)nb, v, vi, m, ov, oi, last, w8, s)) return rc;
        w8 = false;
        v = ov;
        vi = oi;
        uv += nb;
        if (am) ui += nb;
        m = nb;
    }
    return 0;
}

// The fused reduction of root over n elements (inputs resolved by
// `resolve`, halo preceding samples) into value/index; idx_base is the
// index of element 0.
template <class Resolve>
int reduce_fused(const simtgo_tile_graph* g, int root, int kind, int64_t n, int64_t halo,
                 int64_t idx_base, cudaStream_t s, Resolve resolve, float* value, int64_t* index) {
    const bool am = kind == tilek::RED_ARGMAX;
    if (n == 0) return finish_levels(kind, nullptr, nullptr, 0, value, index, s, nullptr, nullptr);
    Lowered L;
    int rc = lower(g, root, L, kind);
    if (rc) return rc;
    std::vector<const float*> dev_in;
    for (int id : L.in_nodes) {
        const float* p = resolve(id);
        if (!p) return sg::fail(SIMTGO_EARG, "tile: input node %d has no device data", id);
        dev_in.push_back(p);
    }
    const int64_t m = n_partials(n);
    const int64_t slots = 8 * m + upper_slots(m);
    AsyncBuf bv, bi;
    if ((rc = bv.alloc(slots * sizeof(float), s))) return rc;
    if (am && (rc = bi.alloc(slots * sizeof(int64_t), s))) return rc;
    float* pv = (float*)bv.p;
    int64_t* pi = (int64_t*)bi.p;
    if ((rc = launch_program(g, L, dev_in, pv, n, halo, s, pi, idx_base))) return rc;
    return finish_levels(kind, pv, pi, m, value, index, s, pv + 8 * m,
                         am ? pi + 8 * m : nullptr);
}

int check_reduce(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind, const void* value,
                 const void* index) {
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    if (!g->err.empty()) return sg::fail(SIMTGO_EGRAPH, "%s", g->err.c_str());
    if (!valid(g, t)) return sg::fail(SIMTGO_EARG, "tile: unknown tensor %d", t);
    if (kind < tilek::RED_SUM || kind > tilek::RED_ARGMAX)
        return sg::fail(SIMTGO_EARG, "tile: unknown reduction %d", kind);
    if (!value) return sg::fail(SIMTGO_ENULL, "tile: null reduction value");
    if (kind == tilek::RED_ARGMAX && !index)
        return sg::fail(SIMTGO_ENULL, "tile: ARGMAX needs an index");
    return 0;
}

}  // namespace

namespace sg {
int comm_rank(const simtgo_comm* c, int* nranks, int* rank);
int comm_allgather(simtgo_comm* c, const void* send, void* recv, size_t bytes, cudaStream_t s);
}  // namespace sg

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
    if (!g->chained && contains_fir(g, a)) {
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

int simtgo_tile_allow_chained_windows(simtgo_tile_graph* g, int32_t allow) {
    sg::clear_error();
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    g->chained = allow != 0;
    return 0;
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
    if (n_instructions) *n_instructions = (int32_t)L.code.size();
    if (n_inputs) *n_inputs = (int32_t)L.in_nodes.size();
    if (n_windows) *n_windows = (int32_t)L.fir_nodes.size();
    return 0;
}

// The listing of a lowered program, one device instruction per line:
//   "window <f> taps <T> node <id>" / "main" section headers, then
//   "<pc> <step> | <step> ...", the steps the instruction fuses, in order:
//   "lda <m>", "add|mul|hypot <m>", "scale <k as %a>", "sqrt", "abs",
//   "firacc w<f>", "sta t<j>", "stage w<f>", "store", "end",
// where an operand <m> is in<k> (input k), t<j> (temporary j), w<f> (the
// signal of window f over the chunk) or acc (the accumulator itself).
static std::string listing(const simtgo_tile_graph* g, const Lowered& L) {
    std::string s;
    char line[256];
    snprintf(line, sizeof line,
             "; simtgo_b200 tile program: %zu instructions, %zu inputs, %zu windows, %d temporaries\n",
             L.code.size(), L.in_nodes.size(), L.fir_nodes.size(), L.n_tmp);
    s += line;
    for (size_t k = 0; k < L.in_nodes.size(); k++) {
        snprintf(line, sizeof line, "; in%zu = node %d (p%d)\n", k, L.in_nodes[k],
                 L.param_of[L.in_nodes[k]]);
        s += line;
    }
    static const char* const names[tilek::OP_KINDS] = {
        "end", "lda", "sta", "add", "mul", "hypot", "scale", "sqrt", "abs", "firacc", "stage", "store"};
    auto operand = [](uint8_t space, int idx) -> std::string {
        char b[32];
        switch (space) {
            case SP_IN: snprintf(b, sizeof b, "in%d", idx); break;
            case SP_TMP: snprintf(b, sizeof b, "t%d", idx); break;
            case SP_WIN: snprintf(b, sizeof b, "w%d", idx); break;
            default: snprintf(b, sizeof b, "acc"); break;
        }
        return b;
    };
    for (size_t pc = 0; pc < L.code.size(); pc++) {
        for (size_t f = 0; f < L.fir_nodes.size(); f++)
            if (L.fir_start[f] == (int32_t)pc) {
                const Node& fn = g->nodes[L.fir_nodes[f]];
                snprintf(line, sizeof line, "window %zu taps %zu node %d\n", f,
                         g->nodes[fn.b].taps.size(), L.fir_nodes[f]);
                s += line;
            }
        if ((int32_t)pc == L.main_start) s += "main\n";
        const FInsn& in = L.code[pc];
        std::vector<std::string> steps;
        if (in.loada) steps.push_back("lda " + operand(in.a_space, in.a_idx));
        if (in.op == tilek::OP_SCALE) {
            snprintf(line, sizeof line, "scale %a", (double)in.imm);
            steps.push_back(line);
        } else if (in.op == tilek::OP_FIRACC) {
            steps.push_back("firacc w" + std::to_string(in.b_idx));
        } else if (in.op == tilek::OP_ADD || in.op == tilek::OP_MUL || in.op == tilek::OP_HYPOT) {
            steps.push_back(std::string(names[in.op]) + " " + operand(in.b_space, in.b_idx));
        } else if (in.op != tilek::OP_END) {
            steps.push_back(names[in.op]);
        }
        if (in.sta) steps.push_back("sta t" + std::to_string(in.d_idx));
        if (in.stage) steps.push_back("stage w" + std::to_string(in.d_idx));
        if (in.store) steps.push_back("store");
        if (in.end) steps.push_back("end");
        std::string text = std::to_string(pc) + " ";
        for (size_t i = 0; i < steps.size(); i++) text += (i ? " | " : "") + steps[i];
        s += text + "\n";
    }
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

int simtgo_tile_reduce(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind, float* dev_value,
                       int64_t* dev_index, void* stream) {
    sg::clear_error();
    int rc;
    if ((rc = check_reduce(g, t, kind, dev_value, dev_index))) return rc;
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    auto resolve = [&](int id) -> const float* { return g->nodes[id].dev; };
    return reduce_fused(g, t, kind, g->nodes[t].n, 0, 0, (cudaStream_t)stream, resolve,
                        dev_value, dev_index);
}

int simtgo_tile_reduce_materialize(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind,
                                   float* value, int64_t* index) {
    sg::clear_error();
    int rc;
    if ((rc = check_reduce(g, t, kind, value, index))) return rc;
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    std::vector<DevBuf> owned;
    std::unordered_map<int, const float*> uploaded;
    DevBuf res;
    if ((rc = sg::cuda_status(cudaMalloc(&res.p, 16), "cudaMalloc"))) return rc;
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
    int64_t* res_i = reinterpret_cast<int64_t*>(res.p + 2);
    rc = reduce_fused(g, t, kind, g->nodes[t].n, 0, 0, 0, resolve, res.p, res_i);
    if (err) return err;
    if (rc) return rc;
    if ((rc = sg::cuda_status(cudaStreamSynchronize(0), "tile reduce"))) return rc;
    if ((rc = sg::cuda_status(cudaMemcpy(value, res.p, sizeof(float), cudaMemcpyDeviceToHost),
                              "download")))
        return rc;
    if (kind == tilek::RED_ARGMAX)
        rc = sg::cuda_status(cudaMemcpy(index, res_i, sizeof(int64_t), cudaMemcpyDeviceToHost),
                             "download");
    return rc;
}

int simtgo_tile_shard_range(int64_t n_total, int32_t nranks, int32_t rank, int64_t* start,
                            int64_t* len) {
    sg::clear_error();
    if (!start || !len) return sg::fail(SIMTGO_ENULL, "tile: null shard range output");
    if (n_total < 0 || nranks < 1 || rank < 0 || rank >= nranks)
        return sg::fail(SIMTGO_EARG, "tile: shard %d of %d over %lld elements", rank, nranks,
                        (long long)n_total);
    const int64_t per = n_partials((n_total + nranks - 1) / nranks) * tilek::kChunk;
    *start = std::min<int64_t>((int64_t)rank * per, n_total);
    *len = std::min<int64_t>(*start + per, n_total) - *start;
    return 0;
}

int simtgo_tile_reduce_shard(simtgo_tile_graph* g, simtgo_tensor t, int32_t kind, int32_t halo,
                             int64_t n_total, simtgo_comm* comm, float* dev_value,
                             int64_t* dev_index, void* stream) {
    sg::clear_error();
    int rc;
    if ((rc = check_reduce(g, t, kind, dev_value, dev_index))) return rc;
    if (halo < 0) return sg::fail(SIMTGO_EARG, "tile: negative halo");
    int nranks, rank;
    if ((rc = sg::comm_rank(comm, &nranks, &rank))) return rc;
    int64_t start, len;
    if ((rc = simtgo_tile_shard_range(n_total, nranks, rank, &start, &len))) return rc;
    if (g->nodes[t].n != len)
        return sg::fail(SIMTGO_ELENGTH,
                        "tile: rank %d of %d holds elements [%lld, %lld) of %lld, the tensor has %d",
                        rank, nranks, (long long)start, (long long)(start + len),
                        (long long)n_total, g->nodes[t].n);
    const sg::DevInfo* d;
    if ((rc = sg::current_device(&d))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    auto resolve = [&](int id) -> const float* { return g->nodes[id].dev; };
    // Every rank takes the same steps: n_total, and so C, are the same on all.
    if (n_total == 0 || nranks == 1)
        return reduce_fused(g, t, kind, len, halo, start, s, resolve, dev_value, dev_index);
    const bool am = kind == tilek::RED_ARGMAX;
    int64_t s0, per;
    if ((rc = simtgo_tile_shard_range(n_total, nranks, 0, &s0, &per))) return rc;
    const int64_t C = 8 * (per / tilek::kChunk);  // warp-partial slots per rank
    const int64_t mine = 8 * n_partials(len);
    const int64_t m = n_partials(n_total);
    const int64_t slots = C + C * nranks + upper_slots(m);
    AsyncBuf bv, bi;
    if ((rc = bv.alloc(slots * sizeof(float), s))) return rc;
    if (am && (rc = bi.alloc(slots * sizeof(int64_t), s))) return rc;
    float* send_v = (float*)bv.p;
    float* recv_v = send_v + C;
    int64_t* send_i = am ? (int64_t*)bi.p : nullptr;
    int64_t* recv_i = am ? send_i + C : nullptr;
    if (len > 0) {
        Lowered L;
        if ((rc = lower(g, t, L, kind))) return rc;
        std::vector<const float*> dev_in;
        for (int id : L.in_nodes) {
            const float* p = resolve(id);
            if (!p) return sg::fail(SIMTGO_EARG, "tile: input node %d has no device data", id);
            dev_in.push_back(p);
        }
        if ((rc = launch_program(g, L, dev_in, send_v, len, halo, s, send_i, start))) return rc;
    }
    if (mine < C) {
        sg::before_launch();
        switch (kind) {
            case tilek::RED_SUM:
                tilek::k_red_fill<tilek::RED_SUM><<<1, tilek::kThreads, 0, s>>>(send_v, send_i, mine, C);
                break;
            case tilek::RED_MIN:
                tilek::k_red_fill<tilek::RED_MIN><<<1, tilek::kThreads, 0, s>>>(send_v, send_i, mine, C);
                break;
            case tilek::RED_MAX:
                tilek::k_red_fill<tilek::RED_MAX><<<1, tilek::kThreads, 0, s>>>(send_v, send_i, mine, C);
                break;
            default:
                tilek::k_red_fill<tilek::RED_ARGMAX><<<1, tilek::kThreads, 0, s>>>(send_v, send_i, mine,
                                                                                  C);
        }
        if ((rc = sg::launch_status("tile reduce"))) return rc;
    }
    if ((rc = sg::comm_allgather(comm, send_v, recv_v, C * sizeof(float), s))) return rc;
    if (am && (rc = sg::comm_allgather(comm, send_i, recv_i, C * sizeof(int64_t), s))) return rc;
    // Ranks hold whole chunks in order, so the first 8 m gathered slots are
    // the warp partials of the whole signal's chunks.
    return finish_levels(kind, recv_v, recv_i, m, dev_value, dev_index, s,
                         recv_v + C * nranks, am ? recv_i + C * nranks : nullptr);
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
