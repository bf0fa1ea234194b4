// tile_kernel.cuh -- the device half of the tile track (included once, by
// tile.cu): the accumulator machine's instruction format and program block,
// the interpreter, the window accumulation, the reduction trees and the
// kernels k_tile (the fused graph over chunks of the signal) and
// k_red_level / k_red_fill (the levels of a reduction above its chunks).
// tile.cu's header describes the design; this file is its device code.
#pragma once
#ifndef __CUDACC_RTC__
#include <stdint.h>
#endif

#include "common.cuh"
#include "exact.cuh"
#include "tma.cuh"

using namespace sgd;

namespace tilek {

constexpr int kThreads = 256;
// Float4 groups per thread (the template parameter G): 4 (kGWide) for
// graphs whose four-group layout still fits two blocks per SM, whose
// dispatch and chunk costs then spread over twice the elements (eight
// chained Muls measured 0.57 -> 0.76 of HBM); 2 otherwise. A window's tile
// holds one chunk of either size.
constexpr int kG = 2;
constexpr int kGWide = 4;
__host__ __device__ constexpr int chunk_of(int G) { return kThreads * 4 * G; }
// 2048: the chunk of G = 2 and the block of the reduction trees, whatever G
// the interpreter runs with.
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
__host__ __device__ constexpr int tile_floats(int head, int chunk = kChunk) { return chunk + head + 4; }
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
__device__ __forceinline__ float4 f4_hypot(float4 a, float4 b) { return hypot_go4(a, b); }
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

// Eight taps i0 .. i0+7 (hva, hvb) on the G groups of the thread, whose
// window float4 at tap i0 (a multiple of 4) is tw[256 k - i0/4]: three
// window loads per group, no predicates. No window value is carried from
// one step to the next: a carried float4 costs four register moves per
// step, a third load one shared load (measured at 2^28: a 31-tap window
// 0.781 -> 0.775 ms).
template <int G>
__device__ __forceinline__ void fir_step8(float (&acc)[G][4], const float4* tw, int i0,
                                          const float (&hva)[4], const float (&hvb)[4]) {
#pragma unroll
    for (int k = 0; k < G; k++) {
        const float4 hi = tw[kThreads * k - i0 / 4];
        const float4 m = tw[kThreads * k - i0 / 4 - 1];
        const float4 lo = tw[kThreads * k - i0 / 4 - 2];
        fir_step<false>(acc[k], m, hi, hva, 4);
        fir_step<false>(acc[k], lo, m, hvb, 4);
    }
}
// The last 1-7 taps, 4 (nk <= 4 of them) at a time.
template <int G>
__device__ __forceinline__ void fir_step4(float (&acc)[G][4], const float4* tw, int i0,
                                          const float (&hv)[4], int nk) {
#pragma unroll
    for (int k = 0; k < G; k++) {
        const float4 hi = tw[kThreads * k - i0 / 4];
        const float4 lo = tw[kThreads * k - i0 / 4 - 1];
        fir_step<true>(acc[k], lo, hi, hv, nk);
    }
}

// Window f accumulated at the thread's positions, its descriptor and taps
// read from shared memory (the interpreter).
template <int G>
__device__ __forceinline__ void fir_acc(float4 (&A)[G], const Ctx& c, int f, int woff4) {
    const int4 fd = c.fir[f];
    const int taps = fd.y & (kSyncAfter - 1);
    const float4* h4 = reinterpret_cast<const float4*>(c.taps_s + f * kMaxTaps);
    const float4* tw = c.S + fd.w + threadIdx.x + fd.z / 4 + woff4;
    float acc[G][4];
#pragma unroll
    for (int k = 0; k < G; k++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[k][j] = 0.0f;
    int i0 = 0;
    for (; i0 + 8 <= taps; i0 += 8) {
        const float4 ha = h4[i0 / 4], hb = h4[i0 / 4 + 1];
        const float hva[4] = {ha.x, ha.y, ha.z, ha.w}, hvb[4] = {hb.x, hb.y, hb.z, hb.w};
        fir_step8<G>(acc, tw, i0, hva, hvb);
    }
    for (; i0 < taps; i0 += 4) {
        const float4 hk = h4[i0 / 4];
        const float hv[4] = {hk.x, hk.y, hk.z, hk.w};
        fir_step4<G>(acc, tw, i0, hv, min(4, taps - i0));
    }
#pragma unroll
    for (int k = 0; k < G; k++) A[k] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
}

// The same accumulation with TAPS and the tile's place compile-time
// constants (a graph's specialised kernel): both loops unroll completely
// and the taps h[] are read from the kernel's parameter block, where each
// is an operand of its FMAs.
template <int G, int TAPS>
__device__ __forceinline__ void fir_acc_static(float4 (&A)[G], const float4* tw, const float* h) {
    float acc[G][4];
#pragma unroll
    for (int k = 0; k < G; k++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[k][j] = 0.0f;
#pragma unroll
    for (int i0 = 0; i0 + 8 <= TAPS; i0 += 8) {
        const float hva[4] = {h[i0], h[i0 + 1], h[i0 + 2], h[i0 + 3]};
        const float hvb[4] = {h[i0 + 4], h[i0 + 5], h[i0 + 6], h[i0 + 7]};
        fir_step8<G>(acc, tw, i0, hva, hvb);
    }
#pragma unroll
    for (int i0 = TAPS / 8 * 8; i0 < TAPS; i0 += 4) {
        const float hv[4] = {h[i0], h[i0 + 1], h[i0 + 2], h[i0 + 3]};
        fir_step4<G>(acc, tw, i0, hv, TAPS - i0 < 4 ? TAPS - i0 : 4);
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

// One instruction of a run (the order of its parts is the format's: load,
// operation, temporary, window tile, output). The hooks give what depends
// on where the program lives: hk.win(in, c, r, A) accumulates the window
// the instruction names (OP_FIRACC), hk.tile_of(in, c) is the float4
// offset of the tile it stages (F_STAGE), hk.imm(in) the SCALE factor, and
// hk.tmp_reg(x) says whether the temporary at x lives in registers
// (hk.tmp_get / tmp_set) instead of shared memory. The
// interpreter's hooks read the program in shared memory, a graph's
// specialised kernel's are compile-time constants and its parameter block.
// In DIRECT mode (BULK false) an input operand is read from HBM at the
// run's positions. Returns true at the program's last instruction.
template <bool BULK, bool FULL, int G, class Hooks>
__device__ __forceinline__ bool exec(const Insn& in, const Hooks& hk, const Ctx& c, const Run& r,
                                     float4 (&A)[G], const int t) {
    // Group k of operand M(x) (inactive groups: A itself, nothing is read).
    auto operand = [&](int x, bool input, int k) -> float4 {
        if (!FULL && !((r.gm >> k) & 1)) return A[k];
        if (!BULK && input) return gload4(c.in[x], r.p0 + 4 * (t + kThreads * k), c);
        if (!input && hk.tmp_reg(x)) return hk.tmp_get(x, k);
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
            for (int k = 0; k < G; k++) A[k] = f4_scale(hk.imm(in), A[k]);
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
            hk.win(in, c, r, A);
            break;
        default:
            break;  // OP_END: no operation
    }
    if (in.flags & (F_STA | F_STAGE | F_STORE | F_END)) {
        if (in.flags & F_STA) {
#pragma unroll
            for (int k = 0; k < G; k++)
                if (FULL || ((r.gm >> k) & 1)) {
                    if (hk.tmp_reg(in.d))
                        hk.tmp_set(in.d, k, A[k]);
                    else
                        c.S[in.d + t + kThreads * k] = A[k];
                }
        }
        if (in.flags & F_STAGE) {
            float4* dst = c.S + hk.tile_of(in, c) + r.sh_st + t;
#pragma unroll
            for (int k = 0; k < G; k++)
                if (FULL || ((r.gm >> k) & 1))
                    dst[kThreads * k] =
                        r.edge ? mask_outside(A[k], r.p0 + 4 * (t + kThreads * k), c) : A[k];
        }
        // A run inside [0, n) with a 16-byte aligned output stores its
        // float4s unchecked; the rest element by element.
        if ((in.flags & F_STORE) && !r.edge && c.vec) {
            float* o = c.out + r.p0 + 4 * t;
#pragma unroll
            for (int k = 0; k < G; k++) st_stream_f4(o + 4 * kThreads * k, A[k]);
        } else if (in.flags & F_STORE) {
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
        if (in.flags & F_END) return true;
    }
    return false;
}

template <int G>
struct InterpHooks {
    __device__ __forceinline__ float imm(const Insn& in) const { return in.imm; }
    __device__ __forceinline__ void win(const Insn& in, const Ctx& c, const Run& r,
                                        float4 (&A)[G]) const {
        fir_acc<G>(A, c, in.b, r.woff4);
    }
    __device__ __forceinline__ int tile_of(const Insn& in, const Ctx& c) const {
        return c.fir[in.d].w;
    }
    __device__ __forceinline__ bool tmp_reg(int) const { return false; }
    __device__ __forceinline__ float4 tmp_get(int, int) const { return float4{}; }
    __device__ __forceinline__ void tmp_set(int, int, float4) const {}
};

// Runs the program from pc until an instruction with F_END, leaving the
// last value in A (which a reduction consumes). Inlined into
// k_tile twice: FULL for runs where all of the thread's groups take part
// (the chunk), and the general form for a window's head run. (Loading the
// next instruction ahead measured slower: it costs more instructions than
// the shared-load latency it hides.)
template <bool BULK, bool FULL, int G>
__device__ __forceinline__ void interpret(const Insn* code, int pc, const Ctx& c, const Run& r,
                                          float4 (&A)[G]) {
    const int t = threadIdx.x;
    // Every program's first step writes A (LDA or FIRACC); a head run's
    // inactive groups read A as their own operand, so it starts defined.
    if (!FULL) {
#pragma unroll
        for (int k = 0; k < G; k++) A[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (;;) {
        const Insn in = code[pc++];
        if (exec<BULK, FULL, G>(in, InterpHooks<G>{}, c, r, A, t)) return;
    }
}

// ---- a graph's specialised kernel ------------------------------------------------
// The same program with every instruction and window descriptor a
// compile-time constant: a generated struct S (one per distinct program,
// compiled at run time for sm_100a) supplies
//   static constexpr Insn code[];       the program (imm unused: SCALE
//                                       factors come from the parameter block)
//   static constexpr FirC fir[];        per window (at least one entry)
//   static constexpr int n_fir, main_start, reduce;
//   static constexpr int temps4, n_tmp;  the temporaries' float4 offset and count
//   static constexpr bool tmp_regs;      temporaries in registers, not shared memory
// and exec() runs each instruction with its operation, flags and
// addresses folded, so nothing is decoded or dispatched at run time, and a
// window's taps are parameter-bank operands of its FMAs. The arithmetic is
// exec()'s and fir_acc_core()'s, the interpreter's own: both produce the
// same bits.
struct FirC {
    int32_t start, taps, head, tile4;  // as FirDesc (taps | kSyncAfter)
};

template <class S, int G, int PC, int TAPS, int WTILE, int DTILE>
struct StaticHooks {
    const Program& P;
    float4 (&T)[kMaxTmp][G];  // the temporaries, when S::tmp_regs
    __device__ __forceinline__ float imm(const Insn&) const { return P.code[PC].imm; }
    __device__ __forceinline__ void win(const Insn& in, const Ctx& c, const Run& r,
                                        float4 (&A)[G]) const {
        fir_acc_static<G, TAPS>(A, c.S + WTILE + threadIdx.x + r.woff4, P.fir[in.b].h);
    }
    __device__ __forceinline__ int tile_of(const Insn&, const Ctx&) const { return DTILE; }
    // A temporary's float4 offset x names slot (x - temps4) / (chunk / 4).
    __device__ __forceinline__ bool tmp_reg(int x) const {
        return S::tmp_regs && x >= S::temps4 && x < S::temps4 + S::n_tmp * (chunk_of(G) / 4);
    }
    __device__ __forceinline__ float4 tmp_get(int x, int k) const {
        return T[(x - S::temps4) / (chunk_of(G) / 4)][k];
    }
    __device__ __forceinline__ void tmp_set(int x, int k, float4 v) const {
        T[(x - S::temps4) / (chunk_of(G) / 4)][k] = v;
    }
};

template <class S, int PC, bool BULK, bool FULL, int G>
__device__ __forceinline__ void interpret_s(const Program& P, const Ctx& c, const Run& r,
                                            float4 (&A)[G], float4 (&T)[kMaxTmp][G]) {
    constexpr Insn in = S::code[PC];
    constexpr int FW = in.op == OP_FIRACC ? in.b : 0;
    constexpr int TAPS = S::fir[FW].taps & (kSyncAfter - 1);
    constexpr int WTILE = S::fir[FW].tile4 + S::fir[FW].head / 4;
    constexpr int DTILE = (in.flags & F_STAGE) ? S::fir[in.d].tile4 : 0;
    (void)exec<BULK, FULL, G>(in, StaticHooks<S, G, PC, TAPS, WTILE, DTILE>{P, T}, c, r, A,
                              (int)threadIdx.x);
    if constexpr (!(in.flags & F_END)) interpret_s<S, PC + 1, BULK, FULL, G>(P, c, r, A, T);
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
// The ARGMAX order as one unsigned key per value: every NaN above
// everything, then the value's order with +0 above -0 (the float's bits
// made monotonic). Ties of the key (the same value, or two NaNs) go to the
// smaller offset, so pairwise choices by (key, offset) choose exactly as
// am_before does.
__device__ __forceinline__ uint32_t am_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return v != v ? 0xffffffffu : ((u >> 31) ? ~u : (u | 0x80000000u));
}
// A thread's eight values (offsets increasing with the index into x, so the
// left of each pair keeps a tie), then the warp butterfly on (key, offset);
// every lane ends with the warp's choice. The value comes back from the key
// (its bits, -0 included), or for a NaN from the lane that holds it.
__device__ __forceinline__ RV32 am_warp32(const RV32 (&x)[8]) {
    uint32_t k[8];
    int32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        k[i] = am_key(x[i].v);
        o[i] = x[i].o;
    }
#pragma unroll
    for (int w = 1; w < 8; w *= 2)
#pragma unroll
        for (int i = 0; i < 8; i += 2 * w)
            if (k[i + w] > k[i]) {
                k[i] = k[i + w];
                o[i] = o[i + w];
            }
    uint32_t K = k[0];
    int32_t O = o[0];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const uint32_t k2 = __shfl_xor_sync(0xffffffffu, K, m);
        const int32_t o2 = __shfl_xor_sync(0xffffffffu, O, m);
        if (k2 > K || (k2 == K && o2 < O)) {
            K = k2;
            O = o2;
        }
    }
    float v;
    if (K != 0xffffffffu) {
        v = __uint_as_float((K >> 31) ? (K & 0x7fffffffu) : ~K);
    } else {  // a NaN: its own bits, from the lane whose values hold offset O
        float c = x[0].v;
#pragma unroll
        for (int i = 1; i < 8; i++)
            if (x[i].o == O) c = x[i].v;
        v = __shfl_sync(0xffffffffu, c, (O >> 2) & 31);
    }
    return {v, O};
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
            const bool full = base + kChunk <= n;  // uniform: no value past n
            if constexpr (KIND == RED_ARGMAX) {
                RV32 x[8];
#pragma unroll
                for (int k = 0; k < 2; k++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int32_t o = 4 * (t + kThreads * k) + e;
                        x[4 * k + e] = RV32{f4_get(A[2 * sb + k], e), o};
                    }
                if (!full) {
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        if (base + x[i].o >= n)
                            x[i] = RV32{__int_as_float((int)0xff800000u), INT32_MAX};
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
                    for (int e = 0; e < 4; e++) x[4 * k + e] = RVal{f4_get(A[2 * sb + k], e), 0};
                if (!full) {
#pragma unroll
                    for (int k = 0; k < 2; k++)
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            if (base + 4 * (t + kThreads * k) + e >= n)
                                x[4 * k + e] = red_identity<KIND>();
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

// ---- the streaming reduction -------------------------------------------------
// A reduction whose value is a chain of steps on ONE input (Scale, Sqrt, Abs,
// and Add or Mul of a value with itself) needs neither shared operands
// nor the interpreter. One warp takes a whole 2048-element block: the eight
// rows that warps 0..7 of the interpreter's block hold (lane l of row w: the
// four positions 4 (32 w + l) and the four 1024 later) come straight from
// HBM, one after another, each reduced by the same thread and butterfly
// trees; the eight row results combine as ((w0 w1)(w2 w3))((w4 w5)(w6 w7)),
// the first level's own step, into the chunk's partial. No block barrier.
constexpr int kMaxSteps = 8;
struct Chain {
    int32_t n;               // steps
    int32_t op[kMaxSteps];   // OP_SCALE, OP_SQRT, OP_ABS, OP_ADD, OP_MUL (x op x)
    float imm[kMaxSteps];    // OP_SCALE's factor
};

template <int G>
__device__ __forceinline__ void apply_chain(const Chain& ch, float4 (&A)[G]) {
    static_assert(G == 2, "the streaming reduction holds two groups per row");
    for (int s = 0; s < ch.n; s++) {
        const float k = ch.imm[s];
        switch (ch.op[s]) {  // uniform: one branch per step for all the thread's values
            case OP_SCALE:
#pragma unroll
                for (int j = 0; j < G; j++) A[j] = f4_scale(k, A[j]);
                break;
            case OP_SQRT:
#pragma unroll
                for (int j = 0; j < G; j++) A[j] = f4_sqrt(A[j]);
                break;
            case OP_ABS:
#pragma unroll
                for (int j = 0; j < G; j++) A[j] = f4_abs(A[j]);
                break;
            case OP_ADD:
#pragma unroll
                for (int j = 0; j < G; j++) A[j] = f4_add(A[j], A[j]);
                break;
            default:  // OP_MUL
#pragma unroll
                for (int j = 0; j < G; j++) A[j] = f4_mul(A[j], A[j]);
                break;
        }
    }
}

// Row w of block b for this lane: positions b*kChunk + 4 (32 w + lane) + j
// and 1024 later; positions at or past n read as 0 (the trees put the
// identity there).
__device__ __forceinline__ void load_row(const float* __restrict__ x, int64_t n, int64_t b, int w,
                                         int lane, float4 (&V)[2]) {
    const int64_t p0 = b * kChunk + 4 * (32 * w + lane);
    if ((b + 1) * kChunk <= n) {  // uniform: a whole block
        V[0] = ld_stream_f4(x + p0);
        V[1] = ld_stream_f4(x + p0 + 4 * kThreads);
        return;
    }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        float f[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int64_t p = p0 + 4 * kThreads * k + j;
            f[j] = p < n ? x[p] : 0.0f;
        }
        V[k] = make_float4(f[0], f[1], f[2], f[3]);
    }
}

// A row's eight values of a SUM/MIN/MAX reduction through the thread tree;
// values at positions past n are the identity.
template <int KIND>
__device__ __forceinline__ float row_thread(const float4 (&V)[2], int64_t p0, int64_t n, bool full) {
    RVal x[8];
#pragma unroll
    for (int k = 0; k < 2; k++)
#pragma unroll
        for (int j = 0; j < 4; j++) x[4 * k + j] = RVal{f4_get(V[k], j), 0};
    if (!full) {
#pragma unroll
        for (int k = 0; k < 2; k++)
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (p0 + 4 * kThreads * k + j >= n) x[4 * k + j] = red_identity<KIND>();
    }
    return red_thread<KIND>(x).v;
}

// A row's ARGMAX: the thread's eight values (their keys' maximum and the
// first of them that has it: offsets grow with the index, so the first is
// the smallest offset), then the warp's largest key and the smallest offset
// among the lanes holding it (two warp reductions), and the value from the
// lane that holds it (its bits, NaN payloads included). (K, O, v) is the
// same on every lane.
__device__ __forceinline__ void row_argmax(const float4 (&V)[2], int w, int lane, int64_t cb,
                                           int64_t n, bool full, uint32_t& K, int32_t& O,
                                           float& v) {
    uint32_t k[8];
    float x[8];
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = 4 * c + j;
            x[i] = f4_get(V[c], j);
            k[i] = am_key(x[i]);
        }
    const int32_t o0 = 4 * (32 * w + lane);  // offset of x[0]; x[4 + j] is 1024 later
    if (!full) {
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (cb + o0 + (i >> 2) * 4 * kThreads + (i & 3) >= n) k[i] = 0;  // below any value
    }
    uint32_t mk = k[0];
#pragma unroll
    for (int i = 1; i < 8; i++) mk = max(mk, k[i]);
    int32_t ob = INT32_MAX;
    float vb = 0.0f;
#pragma unroll
    for (int i = 7; i >= 0; i--)
        if (k[i] == mk && mk != 0) {
            ob = o0 + (i >> 2) * 4 * kThreads + (i & 3);
            vb = x[i];
        }
    K = __reduce_max_sync(0xffffffffu, mk);
    O = (int32_t)__reduce_min_sync(0xffffffffu, mk == K ? (uint32_t)ob : 0xffffffffu);
    v = __shfl_sync(0xffffffffu, vb, (O >> 2) & 31);
    if (K == 0) {  // every position past n: the identity
        O = INT32_MAX;
        v = __int_as_float((int)0xff800000u);
    }
}

// One warp per block b in [gw * per, +per) of the nblk 2048-element blocks of
// x (16-byte aligned), gw its index in the grid; out[b] (and, ARGMAX,
// out_i[b] = idx_base + the position) receive the chunk partials. Rows
// stream through a ring of four register slots, three rows ahead of the
// one being reduced.
// The chain's steps applied to a row: RunChain reads them from the
// parameter block at run time (one uniform branch per step); StaticChain<S>
// has them as compile-time constants (S::n steps, S::op[i]; a reduction's
// specialised kernel, compiled at run time), so a row's steps are
// straight-line code. Both take Scale's factor from the parameter block.
struct RunChain {
    static constexpr int kMinBlocks = 0;  // no minimum: the compiler's own register choice
    __device__ __forceinline__ static void apply(const Chain& ch, float4 (&A)[2]) {
        apply_chain<2>(ch, A);
    }
};
template <class S, int I>
__device__ __forceinline__ void apply_static(const Chain& ch, float4 (&A)[2]) {
    if constexpr (I < S::n) {
        constexpr int op = S::op[I];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            if constexpr (op == OP_SCALE)
                A[j] = f4_scale(ch.imm[I], A[j]);
            else if constexpr (op == OP_SQRT)
                A[j] = f4_sqrt(A[j]);
            else if constexpr (op == OP_ABS)
                A[j] = f4_abs(A[j]);
            else if constexpr (op == OP_ADD)
                A[j] = f4_add(A[j], A[j]);
            else
                A[j] = f4_mul(A[j], A[j]);
        }
        apply_static<S, I + 1>(ch, A);
    }
}
template <class S>
struct StaticChain {
    // Unrolled steps raise the register count; three blocks per SM keep
    // the rows in flight.
    static constexpr int kMinBlocks = 3;
    __device__ __forceinline__ static void apply(const Chain& ch, float4 (&A)[2]) {
        apply_static<S, 0>(ch, A);
    }
};

template <int KIND, class CH = RunChain>
__global__ void __launch_bounds__(kThreads, CH::kMinBlocks) k_red_direct(const float* __restrict__ x, int64_t n,
                                                         int64_t idx_base, const Chain ch,
                                                         float* __restrict__ out,
                                                         int64_t* __restrict__ out_i,
                                                         int64_t nblk, int64_t per) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
    const int64_t b0 = gw * per;
    const int64_t b1 = min(b0 + per, nblk);
    if (b0 >= b1) return;
    float4 R[4][2];  // row w of a block lives in slot w % 4
#pragma unroll
    for (int w = 0; w < 3; w++) load_row(x, n, b0, w, lane, R[w]);
    for (int64_t b = b0; b < b1; b++) {
        const int64_t cb = b * kChunk;
        const bool full = cb + kChunk <= n;
        uint32_t bK = 0;
        int32_t bO = INT32_MAX;
        float bv = __int_as_float((int)0xff800000u);
        float acc01 = 0.0f, acc0123 = 0.0f, acc45 = 0.0f, w0 = 0.0f, w4 = 0.0f, w6 = 0.0f;
        auto r2 = [](float a, float c) { return red2<KIND>(RVal{a, 0}, RVal{c, 0}).v; };
#pragma unroll
        for (int w = 0; w < 8; w++) {
            // Row w + 3 (of this block or the next) into the slot row w - 1 left.
            if (w + 3 < 8)
                load_row(x, n, b, w + 3, lane, R[(w + 3) & 3]);
            else if (b + 1 < b1)
                load_row(x, n, b + 1, w + 3 - 8, lane, R[(w + 3) & 3]);
            float4 (&cur)[2] = R[w & 3];
            CH::apply(ch, cur);
            if constexpr (KIND == RED_ARGMAX) {
                uint32_t K;
                int32_t O;
                float v;
                row_argmax(cur, w, lane, cb, n, full, K, O, v);
                if (K > bK || (K == bK && O < bO)) {
                    bK = K;
                    bO = O;
                    bv = v;
                }
            } else {
                float r = row_thread<KIND>(cur, cb + 4 * (32 * w + lane), n, full);
#pragma unroll
                for (int m = 16; m >= 1; m >>= 1) r = r2(r, __shfl_xor_sync(0xffffffffu, r, m));
                // ((w0 w1)(w2 w3))((w4 w5)(w6 w7)), as the rows arrive.
                switch (w) {
                    case 0: w0 = r; break;
                    case 1: acc01 = r2(w0, r); break;
                    case 2: w0 = r; break;
                    case 3: acc0123 = r2(acc01, r2(w0, r)); break;
                    case 4: w4 = r; break;
                    case 5: acc45 = r2(w4, r); break;
                    case 6: w6 = r; break;
                    default: {
                        const float total = r2(acc0123, r2(acc45, r2(w6, r)));
                        if (lane == 0) out[b] = total;
                    }
                }
            }
        }
        if constexpr (KIND == RED_ARGMAX) {
            if (lane == 0) {
                out[b] = bv;
                out_i[b] = bO == INT32_MAX ? kNoIndex : idx_base + cb + bO;
            }
        }
    }
}

// Chunk e's partial from its eight warp partials, ((w0 w1)(w2 w3))((w4 w5)(w6
// w7)) as the first level computes it: ov[e] (and oi[e]) for e < m.
template <int KIND>
__global__ void k_red_w8(const float* __restrict__ v, const int64_t* __restrict__ vi, int64_t m,
                         float* __restrict__ ov, int64_t* __restrict__ oi) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < m;
         e += (int64_t)gridDim.x * blockDim.x) {
        const RVal r = red_block8<KIND>(v + 8 * e, KIND == RED_ARGMAX ? vi + 8 * e : nullptr);
        ov[e] = r.v;
        if (KIND == RED_ARGMAX) oi[e] = r.i;
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
// per-stage mbarriers, so nst-1 chunks stream in while one is interpreted
// (with nst = 1, a four-group window graph's, the next chunk streams in
// while the SM's other block computes). Requires every input 16-byte
// aligned and halo = 0 mod 4. Otherwise
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
//
// tile_body is the kernel's code for both forms: S = Interp runs the
// program from shared memory (k_tile), any other S is a graph's generated
// struct (interpret_s above) and the body is that graph's kernel.
struct Interp {};
template <class S>
struct is_interp {
    static constexpr bool value = false;
};
template <>
struct is_interp<Interp> {
    static constexpr bool value = true;
};

// A specialised kernel's jobs for one chunk, J = 2f (window f's head run,
// first chunk of a range only), 2f + 1 (window f over the chunk), 2 n_fir
// (the main program): the interpreter's job loop with every descriptor a
// constant.
template <class S, int PC, bool BULK, bool FULL, int G>
__device__ __forceinline__ void run_s(const Program& P, const Ctx& c, const Run& r,
                                      float4 (&A)[G], float4 (&T)[kMaxTmp][G]) {
    if (!FULL) {
#pragma unroll
        for (int k = 0; k < G; k++) A[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    interpret_s<S, PC, BULK, FULL, G>(P, c, r, A, T);
}
template <class S, int J, bool BULK, int G>
__device__ __forceinline__ void jobs_s(const Program& P, const Ctx& cx, int32_t in4, int32_t hs,
                                       int64_t cb, bool first, bool edge, float4 (&A)[G],
                                       float4 (&T)[kMaxTmp][G]) {
    constexpr int NF = S::n_fir;
    const int tid = threadIdx.x;
    Run r;
    r.edge = edge;
    if constexpr (J < 2 * NF) {
        constexpr FirC fd = S::fir[J >> 1];
        constexpr int head4 = fd.head / 4;
        if constexpr (!(J & 1)) {
            r.sh_in = in4 + (hs - fd.head) / 4;
            r.sh_st = 0;
            r.woff4 = -head4;
            r.gm = first && tid < head4 ? 1u : 0u;
            r.p0 = cb - fd.head;
            if (r.gm) run_s<S, fd.start, BULK, false, G>(P, cx, r, A, T);
        } else {
            if (!first && tid >= kThreads - head4) {
                float4* tile = cx.S + fd.tile4;
                const int q = tid - (kThreads - head4);
                tile[q] = tile[chunk_of(G) / 4 + q];
            }
            r.sh_in = in4 + hs / 4;
            r.sh_st = head4;
            r.woff4 = 0;
            r.gm = (1u << G) - 1;
            r.p0 = cb;
            run_s<S, fd.start, BULK, true, G>(P, cx, r, A, T);
            if constexpr (J + 1 == 2 * NF || (fd.taps & kSyncAfter)) __syncthreads();
        }
        jobs_s<S, J + 1, BULK, G>(P, cx, in4, hs, cb, first, edge, A, T);
    } else {
        r.sh_in = in4 + hs / 4;
        r.sh_st = 0;
        r.woff4 = 0;
        r.gm = (1u << G) - 1;
        r.p0 = cb;
        run_s<S, S::main_start, BULK, true, G>(P, cx, r, A, T);
    }
}

template <bool BULK, int G, class S>
__device__ __forceinline__ void tile_body(const Program& P, float* __restrict__ out, int64_t n,
                                          int64_t halo, bool vec, bool in_vec, int32_t hs,
                                          int32_t stages4, int32_t nst, uint32_t* wd,
                                          int64_t* __restrict__ out_idx, int64_t idx_base) {
    constexpr bool SPEC = !is_interp<S>::value;
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
    // The program and its windows in shared memory (a specialised kernel
    // has them as constants and reads its taps from the parameter block).
    if constexpr (!SPEC) {
        for (int i = tid; i < code_cap; i += kThreads)
            code_s[i] = i < P.n_code ? P.code[i] : Insn{OP_END, F_END, 0, 0, 0, 0.0f, 0};
        for (int f = tid; f < P.n_fir; f += kThreads)
            fir_s[f] = make_int4(P.fir[f].start, P.fir[f].taps, P.fir[f].head, P.fir[f].tile4);
        for (int f = 0; f < P.n_fir; f++)
            for (int k = tid; k < kMaxTaps; k += kThreads)
                taps_s[f * kMaxTaps + k] = P.fir[f].h[k];  // zero past taps
    }
    for (int k = tid; k < P.n_in; k += kThreads) in_s[k] = P.in[k];

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
    int nf;
    if constexpr (SPEC)
        nf = S::n_fir;
    else
        nf = P.n_fir;
    // The reduction, read where it is used (a parameter-bank operand for
    // the interpreter, a constant for a specialised kernel).
    auto reduce_kind = [&]() -> int {
        if constexpr (SPEC)
            return S::reduce;
        else
            return P.reduce;
    };
    const bool free_run = nf == 0;
    float4 A[G];  // the last run's values (the main program's, for a reduction)
    float4 T[kMaxTmp][G];  // a specialised kernel's temporaries (S::tmp_regs)
    int s = 0;           // this chunk's stage
    uint32_t phase = 0;  // the parity its mbarrier completes next
    for (int64_t c = c0; c < c1; c++) {
        const int64_t cb = c * CH;
        const bool first = c == c0;
        const bool edge = cb - (int64_t)hs < -halo || cb + CH > n;
        if (BULK) {
            if (!mbar_wait(&bars[s], phase, wd)) {
                // Gave up (the watchdog is raised): let the block's other
                // copies in flight land, each wait bounded, before exiting.
                for (int j = 1; j < nst && c + j < c1; j++) {
                    const int s2 = s + j;
                    mbar_wait(&bars[s2 < nst ? s2 : s2 - nst], s2 < nst ? phase : phase ^ 1u, wd);
                }
                return;
            }
            if (edge) {  // only a chunk at either end of the signal has a ragged span
                const ChunkSpan sp = chunk_span(cb, hs, n, halo, first, CH);
                float* buf = stages + s * stage_floats;
                // The last 0-3 samples of a ragged signal are not a whole
                // 16-byte unit: plain loads.
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
        }
        const int32_t in4 = stages4 + s * (stage_floats / 4);
        if constexpr (SPEC) {
            jobs_s<S, 0, BULK, G>(P, cx, in4, hs, cb, first, edge, A, T);
        } else {
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
        }
        if (reduce_kind() != RED_NONE) {
            const int64_t b0 = c * (G / 2), nb = (n + kChunk - 1) / kChunk;
            float* o = out;
            int64_t* oi = out_idx;
            switch (reduce_kind()) {  // uniform: one branch per chunk
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
        if (BULK && ++s == nst) {
            s = 0;
            phase ^= 1u;
        }
    }
}

template <bool BULK, int G>
__global__ void __launch_bounds__(kThreads, G == kG ? 3 : 2)
    k_tile(const __grid_constant__ Program P, float* __restrict__ out, int64_t n, int64_t halo,
           bool vec, bool in_vec, int32_t hs, int32_t stages4, int32_t nst, uint32_t* wd,
           int64_t* __restrict__ out_idx, int64_t idx_base) {
    tile_body<BULK, G, Interp>(P, out, n, halo, vec, in_vec, hs, stages4, nst, wd, out_idx,
                               idx_base);
}

}  // namespace tilek
