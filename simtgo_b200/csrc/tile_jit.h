// tile_jit.h -- host interface of tile_jit.cu (a tile graph's specialised
// kernel, compiled at run time) for tile.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

#include "tile_kernel.cuh"

namespace tilejit {

// The form of a specialised kernel besides its program: input addressing
// (bulk copies or direct loads), float4 groups per thread, and where the
// temporaries live (registers, tmp_regs, or shared memory at temps4).
struct Form {
    bool bulk;
    int g;
    bool tmp_regs;
    int temps4, n_tmp;
};

// The source of the specialised kernel for program P (instructions and
// window descriptors as constants; inputs, taps and SCALE factors stay in
// the parameter block).
std::string spec_source(const tilek::Program& P, const Form& f);

// The compiled kernel for P on the current device (compiled and cached on
// first use, its dynamic shared memory limit set to dyn_max), or nullptr
// with 0 when specialisation is off or (mode 1) NVRTC is unavailable.
int get(const tilek::Program& P, const Form& f, int dyn_max, CUfunction* out);

// The streaming reduction k_red_direct<kind> with the chain ch's steps as
// constants (compiled and cached like get); nullptr with 0 when
// specialisation is off or unavailable.
int get_chain(int kind, const tilek::Chain& ch, CUfunction* out);
// Its source (and the kernel's name expression), and a compile without
// loading (no GPU needed).
std::string chain_source(int kind, const tilek::Chain& ch, std::string* expr);
int compile_chain_only(int kind, const tilek::Chain& ch);

// Whether launches use specialised kernels (mode != 0 and NVRTC and the
// driver's module entry points are there; always true in mode 2).
bool available();

// Resident blocks per SM of fn at kThreads threads and smem bytes.
int occupancy(CUfunction fn, size_t smem, int* blocks);

// Launches fn (the k_tile parameter list in args) on stream s.
int launch(CUfunction fn, int blocks, size_t smem, cudaStream_t s, void** args);

// Compiles the specialised source of P without loading it (no GPU needed).
int compile_only(const tilek::Program& P, const Form& f);

}  // namespace tilejit
