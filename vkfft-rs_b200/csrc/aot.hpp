// Ahead-of-time specialised pass kernels.
//
// The op-program interpreter (kernels.cu) reads every size, stride and radix of a generic
// pass from its parameters.  A specialised kernel of the same pass has the pass's
// structure as compile-time constants -- the CTA's thread count, lines per CTA, the
// shared-memory layout, every op's kind, radix, sub-line lengths, bases, strides and fast
// divisors, the sides' masking and Hermitian fields -- so index arithmetic folds and every
// op loop has a constant stride and trip bound (the compiler unrolls the rounds of a radix
// stage and overlaps their loads).  What differs between two tensors with the same line
// structure stays a run-time parameter: the number of lines, the line decomposition, the
// sides' outer / line / column strides (and the element stride unless it is 1), the
// scales, table offsets and every pointer.
//
// The build lowers a catalogue of transforms (gen_aot.cpp), emits one kernel per distinct
// structure key and compiles them for sm_100a into the library; each registers itself
// under its key at load time.  A pass whose key is in the catalogue runs its specialised
// kernel, any other pass the interpreter.  No compiler runs at execution time.
#pragma once

#include <string>
#include <vector>

#include "program.hpp"

namespace b200fft {

// Structure key of a generic pass (KERNEL_PASS): the compile-time fields of its
// specialised kernel, in a canonical text form.
std::string aot_pass_key(const PassPlan &pp, int scalar_kind);

// CUDA source of the specialised kernel `name` of a generic pass (for the build's
// generator); B200FFT_NT must be defined to pp.threads in the translation unit.
std::string aot_pass_source(const PassPlan &pp, int scalar_kind, const std::string &name);

// Registration of a compiled kernel under its key (called from the generated units'
// static initialisers).
void aot_register(const char *key, const void *fn);

// Per pass of a program: its specialised kernel, or null (interpreter).  Opts the kernels
// in to the full dynamic shared memory on `device` (the current device).
std::vector<const void *> aot_kernels_for(const Program &prog, int device);

// Number of generic passes of a program, and how many of them have a specialised kernel.
int aot_coverage(const Program &prog, int *generic_passes);

}  // namespace b200fft
