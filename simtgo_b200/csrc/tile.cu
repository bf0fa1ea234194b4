// tile.cu -- the tile track (package tile): graph recording (tile/tile.go),
// lowering to one fused program (tile/codegen.go) and running it
// (tile/run.go).
//
// The reference renders each graph as CUDA C and compiles it with NVRTC per
// distinct graph (tile/run.go:40). Here the graph is lowered on the host to a
// short program for an accumulator machine that travels in the kernel's
// parameter block. A precompiled sm_100a kernel interprets it, and by
// default the program runs instead in its own specialised kernel
// (tile_jit.cu): the same kernel body with the program compiled in as
// constants. The machine:
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
#include "tile_jit.h"
#include "tile_kernel.cuh"
#include "tma.cuh"

using namespace sgd;

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
int32_t tile_off4(const Lowered& L, int f, int chunk) {
    int32_t off = 0;
    for (int i = 0; i < f; i++) off += tilek::tile_floats(L.head[i], chunk) / 4;
    return off;
}

// The launch's shared-memory layout (float4 offsets) and its program.
struct Layout {
    int32_t taps4, tiles4, temps4, stages4, sstride, nst;
    int32_t g;  // float4 groups per thread (the interpreter's G); chunk = 1024 g
    size_t smem;
};

// Floats per thread a specialised kernel may hold its temporaries in
// (registers); programs with more keep them in shared memory.
constexpr int kTmpRegFloats = 32;

// Device instructions up to which a program gets a specialised kernel;
// longer ones run on the interpreter (whose dispatch cost they amortise over
// more work). Compile time grows faster than the length: measured 0.7 s at
// 9 instructions, 1.3 s at 18, 2.6 s at 30, 4.8 s at 42, 14 s at 75, and
// from a few hundred on NVRTC refuses the template recursion.
constexpr int kMaxSpecCode = 32;

// The float4 offsets of the layout's parts for Y.g groups per thread; hs
// is the samples a chunk's windows reach below it.
void set_offsets(const Lowered& L, int32_t hs, Layout& Y) {
    const int n_in = (int)L.in_nodes.size(), n_fir = (int)L.fir_nodes.size();
    const int chunk = tilek::chunk_of(Y.g);
    Y.taps4 = tilek::meta_bytes((int)L.code.size(), n_in, n_fir) / 16;
    Y.tiles4 = Y.taps4 + n_fir * tilek::kMaxTaps / 4;
    Y.temps4 = Y.tiles4 + tile_off4(L, n_fir, chunk);
    Y.stages4 = Y.temps4 + L.n_tmp * chunk / 4;
    Y.sstride = hs + chunk;
}

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
        P.fir[f].tile4 = Y.tiles4 + tile_off4(L, f, tilek::chunk_of(Y.g));
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
                   cudaStream_t s, int64_t* out_idx = nullptr, int64_t idx_base = 0,
                   bool jit_ok = true) {
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
    // Four groups per thread (4096-element chunks: each dispatch and each
    // chunk's pipeline spread over twice the elements) whenever the
    // four-group layout with one input stage leaves room for two blocks per
    // SM; two groups otherwise. A graph with windows may then run with a
    // single stage per block: its next chunk's inputs stream in while the
    // SM's other block computes (measured at 2^28: the twelve-node graph
    // 1.82 -> 1.71 ms, a 31-tap window over one input 1.00 -> 0.85 ms; with
    // two stages required, three inputs and a window fit one block per SM
    // and ran 2.90 ms).
    //
    // A specialised kernel keeps the program's temporaries in registers
    // when they take at most kTmpRegFloats per thread (each is the thread's
    // G float4 groups), and then reserves no shared memory for them.
    const bool jit_on = jit_ok && (int)L.code.size() <= kMaxSpecCode && tilejit::available();
    auto tmp_regs = [&](int g) {
        return jit_on && L.n_tmp > 0 && L.n_tmp * g * 4 <= kTmpRegFloats;
    };
    // A specialised kernel with windows takes four groups only when two
    // input stages still fit two blocks per SM (double-buffered chunks
    // matter more once dispatch costs nothing: the twelve-node graph at 2^28
    // measured 0.88 ms with two groups, three blocks and two stages per SM,
    // against 1.08 ms with four groups and one stage; a 31-tap window over
    // one input keeps four groups, 0.43 ms).
    auto smem_for = [&](int g, int stages) {
        const int ch = tilek::chunk_of(g);
        const size_t fixed = (size_t)tilek::meta_bytes((int)L.code.size(), n_in, n_fir) +
                             (size_t)n_fir * tilek::kMaxTaps * 4 + (size_t)tile_off4(L, n_fir, ch) * 16 +
                             (tmp_regs(g) ? 0 : (size_t)L.n_tmp * ch * 4);
        return fixed + stages * (size_t)n_in * (hs + ch) * sizeof(float);
    };
    const int wide_stages = jit_on ? 2 : 1;
    Y.g = (n_fir == 0 ||
           smem_for(tilek::kGWide, wide_stages) <= (size_t)d->smem_per_sm / 2 - 2048)
              ? tilek::kGWide
              : tilek::kG;
    // Input stages per block.
    const int min_st = Y.g == tilek::kGWide && n_fir > 0 && !jit_on ? 1 : 2;
    set_offsets(L, hs, Y);
    if (tmp_regs(Y.g)) Y.stages4 = Y.temps4;
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
    //
    // The program runs in its specialised kernel (tile_jit.cu: this
    // program's instructions compiled in as constants) when run-time
    // compilation is on, else in the interpreter; the choice of stages
    // follows the registers of the kernel that runs.
    const bool bulk_cand = in_aligned && halo % 4 == 0 && n_in > 0;
    static thread_local tilek::Program P;
    build_program(g, L, Y, bulk_cand, P);
    CUfunction spec = nullptr;
    tilejit::Form form{bulk_cand, Y.g, tmp_regs(Y.g), Y.temps4, L.n_tmp};
    if (jit_on && (rc = tilejit::get(P, form, dyn_max, &spec))) return rc;
    if (!spec && tmp_regs(Y.g)) return sg::fail(SIMTGO_EDEVICE, "tile: no specialised kernel");
    int reg_blocks = 0;
    if (spec) {
        rc = tilejit::occupancy(spec, base_smem, &reg_blocks);
    } else {
        rc = sg::cuda_status(
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &reg_blocks, Y.g == kG ? tilek::k_tile<true, kG> : tilek::k_tile<true, kGWide>,
                tilek::kThreads, base_smem),
            "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile)");
    }
    if (rc) return rc;
    bool bulk = false;
    Y.nst = 0;
    if (bulk_cand) {
        int64_t best_inflight = -1;
        for (int per_sm = std::max(1, reg_blocks); per_sm >= 1; per_sm--) {
            const int64_t share =
                std::min<int64_t>(dyn_max, d->smem_per_sm / per_sm - 2048);
            const int64_t fit = (share - (int64_t)base_smem) / (int64_t)stage_bytes;
            const int nst = (int)std::min<int64_t>(fit, tilek::kMaxStages);
            if (nst < min_st) continue;
            const int64_t inflight = (int64_t)per_sm * std::max(1, nst - 1) * (int64_t)stage_bytes;
            if (inflight > best_inflight) {
                best_inflight = inflight;
                Y.nst = nst;
            }
            if (inflight >= 64 * 1024) {
                Y.nst = nst;
                break;
            }
        }
        bulk = Y.nst >= min_st;
    }
    Y.smem = bulk ? base_smem + Y.nst * stage_bytes : base_smem;
    if (Y.smem > (size_t)dyn_max)
        return sg::fail(SIMTGO_ESIZE, "tile: the program needs %zu bytes of shared memory (max %d)",
                        Y.smem, dyn_max);
    if (bulk != bulk_cand) {  // no room for the stages after all: DIRECT addressing
        build_program(g, L, Y, bulk, P);
        spec = nullptr;
        form.bulk = bulk;
        if (jit_on && (rc = tilejit::get(P, form, dyn_max, &spec))) return rc;
    }
    for (int k = 0; k < n_in; k++) P.in[k] = dev_in[k];  // element 0; [-halo, 0) precede it
    auto kern = Y.g == kG ? (bulk ? tilek::k_tile<true, kG> : tilek::k_tile<false, kG>)
                          : (bulk ? tilek::k_tile<true, kGWide> : tilek::k_tile<false, kGWide>);
    int per_sm = 0;
    if (spec)
        rc = tilejit::occupancy(spec, Y.smem, &per_sm);
    else
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
    const int64_t chunks = sg::ceil_div(n, (int64_t)tilek::chunk_of(Y.g));
    const int64_t resident = (int64_t)d->sms * std::max(1, per_sm);
    const int64_t waves = std::max<int64_t>(1, std::min<int64_t>(8, chunks / (32 * resident)));
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(chunks, waves * resident));
    sg::before_launch();
    uint32_t* wd = sg::watchdog_device_ptr();
    if (spec) {
        bool out_vec = vec, in_vec = in_aligned;
        void* args[] = {&P, &out, &n, &halo, &out_vec, &in_vec, &hs,
                        &Y.stages4, &Y.nst, &wd, &out_idx, &idx_base};
        return tilejit::launch(spec, blocks, Y.smem, s, args);
    }
    kern<<<blocks, tilek::kThreads, Y.smem, s>>>(P, out, n, halo, vec, in_aligned, hs, Y.stages4,
                                                 Y.nst, wd, out_idx, idx_base);
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
// (node id -> device pointer). jit_ok false keeps it on the interpreter
// (loading a specialised kernel's module allocates device memory).
template <class Resolve>
int run_fused(const simtgo_tile_graph* g, int root, float* out, int64_t n, int64_t halo,
              cudaStream_t s, Resolve resolve, bool check_alias, bool jit_ok = true) {
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
    return launch_program(g, L, dev_in, out, n, halo, s, nullptr, 0, jit_ok);
}

// ---- reductions ----------------------------------------------------------------

// Stream-ordered device scratch, released on its stream when it goes out of
// scope (after everything enqueued before).
// The reductions' stream-ordered scratch comes from a pool of the library's
// own per device, which keeps up to 1 GiB of freed memory mapped (the
// default pool returns it at every synchronisation, and mapping it again
// costs more than a 2^28-element reduction).
std::mutex g_pool_mu;
cudaMemPool_t g_pool[64];

int scratch_pool(cudaMemPool_t* out) {
    int dev = -1;
    int rc = sg::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return sg::fail(SIMTGO_EDEVICE, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pool[dev]) {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool;
        if ((rc = sg::cuda_status(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate")))
            return rc;
        uint64_t keep = 1ull << 30;
        if ((rc = sg::cuda_status(
                 cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep),
                 "cudaMemPoolSetAttribute"))) {
            cudaMemPoolDestroy(pool);
            return rc;
        }
        g_pool[dev] = pool;
    }
    *out = g_pool[dev];
    return 0;
}

}  // namespace

namespace sg {
int tile_pool_release() {
    std::lock_guard<std::mutex> lk(g_pool_mu);
    for (int dev = 0; dev < 64; dev++)
        if (g_pool[dev]) {
            const int rc = cuda_status(cudaMemPoolTrimTo(g_pool[dev], 0), "cudaMemPoolTrimTo");
            if (rc) return rc;
        }
    return 0;
}
}  // namespace sg

namespace {

struct AsyncBuf {
    void* p = nullptr;
    cudaStream_t s = 0;
    ~AsyncBuf() {
        if (p) cudaFreeAsync(p, s);
    }
    int alloc(size_t bytes, cudaStream_t st) {
        s = st;
        cudaMemPool_t pool;
        if (int rc = scratch_pool(&pool)) return rc;
        return sg::cuda_status(cudaMallocFromPoolAsync(&p, std::max<size_t>(bytes, 16), pool, st),
                               "cudaMallocFromPoolAsync");
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
// output), 8 m entries; or, with w8 false, one partial per chunk.
int finish_levels(int kind, const float* v, const int64_t* vi, int64_t m, float* value,
                  int64_t* index, cudaStream_t s, float* uv, int64_t* ui, bool w8 = true) {
    const bool am = kind == tilek::RED_ARGMAX;
    if (m <= 1) return red_level(kind, 1, v, vi, m, value, am ? index : nullptr, true, w8, s);
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

// The reduction's value as a chain of steps on one input (the streaming
// path, tilek::k_red_direct): every node from the root down is Scale, Sqrt,
// Abs, or Add/Mul with both operands the same node, ending at one
// device input. False for anything else (windows, two inputs, more than
// kMaxSteps steps).
bool direct_chain(const simtgo_tile_graph* g, int root, tilek::Chain& ch, int& input) {
    int ops[tilek::kMaxSteps];
    float imm[tilek::kMaxSteps];
    int k = 0;
    for (int id = root;;) {
        const Node& nd = g->nodes[id];
        if (nd.kind == K_INPUT) {
            if (nd.is_taps) return false;
            input = id;
            break;
        }
        if (k == tilek::kMaxSteps) return false;
        imm[k] = 0.0f;
        switch (nd.kind) {
            case K_SCALE: ops[k] = tilek::OP_SCALE; imm[k] = nd.scale; break;
            case K_SQRT: ops[k] = tilek::OP_SQRT; break;
            case K_ABS: ops[k] = tilek::OP_ABS; break;
            case K_ADD: ops[k] = tilek::OP_ADD; break;
            case K_MUL: ops[k] = tilek::OP_MUL; break;
            default: return false;  // a window, or Hypot (its float64 registers would slow the rest)
        }
        if ((nd.kind == K_ADD || nd.kind == K_MUL) && nd.b != nd.a)
            return false;
        k++;
        id = nd.a;
    }
    ch.n = k;
    for (int i = 0; i < k; i++) {  // the input's step first
        ch.op[i] = ops[k - 1 - i];
        ch.imm[i] = imm[k - 1 - i];
    }
    return true;
}

// Resident blocks per SM of k_red_direct<kind> (the same on every B200),
// found once.
int direct_blocks_per_sm(int kind, int* out) {
    static std::atomic<int> cache[4];
    int v = cache[kind & 3].load(std::memory_order_relaxed);
    if (v == 0) {
        using namespace tilek;
        cudaError_t e;
        switch (kind) {
            case RED_SUM: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_red_direct<RED_SUM>, kThreads, 0); break;
            case RED_MIN: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_red_direct<RED_MIN>, kThreads, 0); break;
            case RED_MAX: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_red_direct<RED_MAX>, kThreads, 0); break;
            default: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k_red_direct<RED_ARGMAX>, kThreads, 0);
        }
        if (e != cudaSuccess)
            return sg::cuda_status(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(tile reduce)");
        v = std::max(1, v);
        cache[kind & 3].store(v, std::memory_order_relaxed);
    }
    *out = v;
    return 0;
}

// Folds the eight warp partials of each of m chunks (wv/wi, 8 m entries)
// into the chunk partials pv/pi (m entries).
int fold_warps(int kind, const float* wv, const int64_t* wi, int64_t m, float* pv, int64_t* pi,
               cudaStream_t s) {
    using namespace tilek;
    if (m <= 0) return 0;
    const unsigned fb = (unsigned)std::min<int64_t>(sg::ceil_div(m, (int64_t)kThreads), 1024);
    sg::before_launch();
    switch (kind) {
        case RED_SUM: k_red_w8<RED_SUM><<<fb, kThreads, 0, s>>>(wv, wi, m, pv, pi); break;
        case RED_MIN: k_red_w8<RED_MIN><<<fb, kThreads, 0, s>>>(wv, wi, m, pv, pi); break;
        case RED_MAX: k_red_w8<RED_MAX><<<fb, kThreads, 0, s>>>(wv, wi, m, pv, pi); break;
        default: k_red_w8<RED_ARGMAX><<<fb, kThreads, 0, s>>>(wv, wi, m, pv, pi);
    }
    return sg::launch_status("tile reduce");
}

// The partial of every 2048-element chunk of root's value over n elements
// (inputs resolved by `resolve`, halo preceding samples) into pv/pi,
// ceil(n/2048) entries; idx_base is the index of element 0. A chain of steps
// on one aligned input streams through k_red_direct (one warp per chunk);
// any other graph runs the interpreter, whose eight warp partials per chunk
// (in wv/wi, 8 ceil(n/2048) entries of scratch) are then folded. Both give
// the same bits: the same trees in the same order.
template <class Resolve>
int launch_partials(const simtgo_tile_graph* g, int root, int kind, int64_t n, int64_t halo,
                    int64_t idx_base, cudaStream_t s, Resolve resolve, float* pv, int64_t* pi,
                    float* wv, int64_t* wi) {
    tilek::Chain ch;
    int input = -1;
    int rc;
    const int64_t nblk = n_partials(n);
    if (direct_chain(g, root, ch, input)) {
        const float* x = resolve(input);
        if (!x) return sg::fail(SIMTGO_EARG, "tile: input node %d has no device data", input);
        if (sg::aligned16(x)) {
            const sg::DevInfo* d;
            if ((rc = sg::current_device(&d))) return rc;
            // One wave of resident blocks; each warp takes a contiguous
            // range of chunks.
            // A chain with steps, and any ArgMax, runs in the reduction's
            // specialised kernel (the steps compiled in as constants:
            // straight-line code per row) when run-time compilation is on:
            // measured at 2^28, ArgMax(Abs(Scale(a, k))) 0.54 -> 0.205 ms,
            // Max(Abs(a)) 0.250 -> 0.195, Sum(Sqrt(Abs(a))) 0.390 -> 0.216,
            // Sum(a*a) 0.176 -> 0.170, ArgMax(a) 0.212 -> 0.183 (the run-time
            // chain's branch per step and row held the rows' loads back);
            // Sum(a) and Max(a), with no step, stay on the precompiled
            // kernel (0.170 and 0.185 there, 0.175 and 0.197 specialised).
            CUfunction spec = nullptr;
            if ((ch.n > 0 || kind == tilek::RED_ARGMAX) && tilejit::available() &&
                (rc = tilejit::get_chain(kind, ch, &spec)))
                return rc;
            int ps;
            if (spec)
                rc = tilejit::occupancy(spec, 0, &ps);
            else
                rc = direct_blocks_per_sm(kind, &ps);
            if (rc) return rc;
            ps = std::max(1, ps);
            const int64_t warps = (int64_t)d->sms * ps * (tilek::kThreads / 32);
            const int64_t per = sg::ceil_div(nblk, std::min<int64_t>(nblk, warps));
            const int64_t used = sg::ceil_div(nblk, per);
            const unsigned blocks = (unsigned)sg::ceil_div(used, (int64_t)(tilek::kThreads / 32));
            sg::before_launch();
            if (spec) {
                int64_t nn = n, ib = idx_base, nb = nblk, pp = per;
                const float* xx = x;
                void* args[] = {&xx, &nn, &ib, &ch, &pv, &pi, &nb, &pp};
                return tilejit::launch(spec, (int)blocks, 0, s, args);
            }
            using namespace tilek;
            switch (kind) {
                case RED_SUM: k_red_direct<RED_SUM><<<blocks, kThreads, 0, s>>>(x, n, idx_base, ch, pv, pi, nblk, per); break;
                case RED_MIN: k_red_direct<RED_MIN><<<blocks, kThreads, 0, s>>>(x, n, idx_base, ch, pv, pi, nblk, per); break;
                case RED_MAX: k_red_direct<RED_MAX><<<blocks, kThreads, 0, s>>>(x, n, idx_base, ch, pv, pi, nblk, per); break;
                default: k_red_direct<RED_ARGMAX><<<blocks, kThreads, 0, s>>>(x, n, idx_base, ch, pv, pi, nblk, per);
            }
            return sg::launch_status("tile reduce (streaming)");
        }
    }
    Lowered L;
    if ((rc = lower(g, root, L, kind))) return rc;
    std::vector<const float*> dev_in;
    for (int id : L.in_nodes) {
        const float* p = resolve(id);
        if (!p) return sg::fail(SIMTGO_EARG, "tile: input node %d has no device data", id);
        dev_in.push_back(p);
    }
    if ((rc = launch_program(g, L, dev_in, wv, n, halo, s, wi, idx_base))) return rc;
    return fold_warps(kind, wv, wi, nblk, pv, pi, s);
}

// The fused reduction of root over n elements (inputs resolved by
// `resolve`, halo preceding samples) into value/index; idx_base is the
// index of element 0.
template <class Resolve>
int reduce_fused(const simtgo_tile_graph* g, int root, int kind, int64_t n, int64_t halo,
                 int64_t idx_base, cudaStream_t s, Resolve resolve, float* value, int64_t* index) {
    const bool am = kind == tilek::RED_ARGMAX;
    if (n == 0) return finish_levels(kind, nullptr, nullptr, 0, value, index, s, nullptr, nullptr);
    int rc;
    const int64_t m = n_partials(n);
    // m chunk partials, the levels above them, and 8 m warp partials of
    // scratch for the interpreter's path.
    const int64_t slots = m + upper_slots(m) + 8 * m;
    AsyncBuf bv, bi;
    if ((rc = bv.alloc(slots * sizeof(float), s))) return rc;
    if (am && (rc = bi.alloc(slots * sizeof(int64_t), s))) return rc;
    float* pv = (float*)bv.p;
    int64_t* pi = (int64_t*)bi.p;
    float* uv = pv + m;
    int64_t* ui = am ? pi + m : nullptr;
    float* wv = uv + upper_slots(m);
    int64_t* wi = am ? ui + upper_slots(m) : nullptr;
    if ((rc = launch_partials(g, root, kind, n, halo, idx_base, s, resolve, pv, pi, wv, wi)))
        return rc;
    return finish_levels(kind, pv, pi, m, value, index, s, uv, ui, false);
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

// The specialised kernel's source for t (reduced by `reduce`, or -1) with
// `groups` float4 groups per thread and bulk or DIRECT input addressing,
// into buf like simtgo_tile_source; with compile != 0 it is also compiled
// (no GPU needed) and a compilation error is returned.
int32_t simtgo_tile_jit_source(simtgo_tile_graph* g, simtgo_tensor t, int32_t reduce,
                               int32_t groups, int32_t bulk, int32_t compile, char* buf,
                               int32_t cap) {
    sg::clear_error();
    if (!g) return sg::fail(SIMTGO_ENULL, "tile: null graph");
    if (!g->err.empty()) return sg::fail(SIMTGO_EGRAPH, "%s", g->err.c_str());
    if (!valid(g, t)) return sg::fail(SIMTGO_EARG, "tile: unknown tensor %d", t);
    if (reduce < -1 || reduce > SIMTGO_TILE_ARGMAX)
        return sg::fail(SIMTGO_EARG, "tile: unknown reduction %d", (int)reduce);
    auto give = [&](const std::string& s) {
        if (buf && cap > 0) {
            const size_t n = std::min<size_t>(s.size(), (size_t)cap - 1);
            memcpy(buf, s.data(), n);
            buf[n] = 0;
        }
        return (int32_t)s.size() + 1;
    };
    int rc;
    if (groups == 0) {  // the streaming reduction of a chain on one input
        tilek::Chain ch;
        int input = -1;
        if (reduce < 0 || !direct_chain(g, t, ch, input))
            return sg::fail(SIMTGO_EARG,
                            "tile: groups 0 names the streaming reduction, which takes a "
                            "reduction of a chain of steps on one input");
        if (compile && (rc = tilejit::compile_chain_only(reduce, ch))) return rc;
        std::string expr;
        return give(tilejit::chain_source(reduce, ch, &expr));
    }
    if (groups != tilek::kG && groups != tilek::kGWide)
        return sg::fail(SIMTGO_EARG, "tile: %d groups per thread is not 0, %d or %d",
                        (int)groups, tilek::kG, tilek::kGWide);
    Lowered L;
    if ((rc = lower(g, t, L, reduce))) return rc;
    int32_t hs = 0;
    for (size_t f = 0; f < L.fir_nodes.size(); f++) hs = std::max<int32_t>(hs, L.head[f]);
    Layout Y{};
    Y.g = groups;
    set_offsets(L, hs, Y);
    static thread_local tilek::Program P;
    build_program(g, L, Y, bulk != 0, P);
    const tilejit::Form form{bulk != 0, (int)groups,
                             L.n_tmp > 0 && L.n_tmp * groups * 4 <= kTmpRegFloats, Y.temps4,
                             L.n_tmp};
    if (compile && (rc = tilejit::compile_only(P, form))) return rc;
    return give(tilejit::spec_source(P, form));
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
    // Each rank exchanges one partial per chunk (launch_partials), so the
    // all-gather moves one float (and one index) per 2048 elements.
    // Chunk-partial slots per rank: rank 0 holds the most chunks (whole ones,
    // unless it holds the entire signal).
    const int64_t C = n_partials(per);
    const int64_t mine = n_partials(len);
    const int64_t m = n_partials(n_total);
    const int64_t slots = C + C * nranks + upper_slots(m) + 8 * mine;
    AsyncBuf bv, bi;
    if ((rc = bv.alloc(slots * sizeof(float), s))) return rc;
    if (am && (rc = bi.alloc(slots * sizeof(int64_t), s))) return rc;
    float* send_v = (float*)bv.p;
    float* recv_v = send_v + C;
    float* warp_v = recv_v + C * nranks + upper_slots(m);
    int64_t* send_i = am ? (int64_t*)bi.p : nullptr;
    int64_t* recv_i = am ? send_i + C : nullptr;
    int64_t* warp_i = am ? recv_i + C * nranks + upper_slots(m) : nullptr;
    using namespace tilek;
    if (len > 0 && (rc = launch_partials(g, t, kind, len, halo, start, s, resolve, send_v, send_i,
                                         warp_v, warp_i)))
        return rc;
    if (mine < C) {
        sg::before_launch();
        switch (kind) {
            case RED_SUM: k_red_fill<RED_SUM><<<1, kThreads, 0, s>>>(send_v, send_i, mine, C); break;
            case RED_MIN: k_red_fill<RED_MIN><<<1, kThreads, 0, s>>>(send_v, send_i, mine, C); break;
            case RED_MAX: k_red_fill<RED_MAX><<<1, kThreads, 0, s>>>(send_v, send_i, mine, C); break;
            default: k_red_fill<RED_ARGMAX><<<1, kThreads, 0, s>>>(send_v, send_i, mine, C);
        }
        if ((rc = sg::launch_status("tile reduce"))) return rc;
    }
    if ((rc = sg::comm_allgather(comm, send_v, recv_v, C * sizeof(float), s))) return rc;
    if (am && (rc = sg::comm_allgather(comm, send_i, recv_i, C * sizeof(int64_t), s))) return rc;
    // Ranks hold whole chunks in order, so the first m gathered slots are
    // the partials of the whole signal's chunks.
    return finish_levels(kind, recv_v, recv_i, m, dev_value, dev_index, s, recv_v + C * nranks,
                         am ? recv_i + C * nranks : nullptr, false);
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
    if (g->nodes[t].kind == K_INPUT) {
        // The root is an input: its values are copied to dev_out by the same
        // one-node program simtgo_tile_run launches (after the same alias check).
        auto resolve = [&](int nid) -> const float* { return g->nodes[nid].dev; };
        return run_fused(g, t, dev_out, out_len, 0, (cudaStream_t)stream, resolve, true, false);
    }
    auto value = [&](int id) -> const float* {
        return g->nodes[id].kind == K_INPUT ? g->nodes[id].dev : scratch + region[id];
    };
    for (int id : order) {
        const Node& nd = g->nodes[id];
        if (nd.kind == K_INPUT) continue;
        simtgo_tile_graph one;
        const int a = simtgo_tile_input_device(&one, value(nd.a), g->nodes[nd.a].n);
        int r = a;
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
        // A step the one-node graph refused comes back as its recorded error,
        // never as a node index.
        if (r < 0 || !one.err.empty())
            return sg::fail(SIMTGO_EGRAPH, "tile: step for node %d: %s", id,
                            one.err.empty() ? "refused" : one.err.c_str());
        float* target = id == t ? dev_out : scratch + region[id];
        auto resolve = [&](int nid) -> const float* { return one.nodes[nid].dev; };
        rc = run_fused(&one, r, target, nd.n, 0, (cudaStream_t)stream, resolve, true, false);
        if (rc) return rc;
    }
    return 0;
}

extern "C" {

}  // extern "C"
