// Persistent frame kernel (frame.cu): a list of decode-frame phases in one
// cooperative, clustered launch with grid barriers between phases.  In the
// device copy of a program, Phase::pad of every phase holds the index of the
// next GEMM phase (-1: none), which the weight prefetch follows.
#pragma once
#include "lm_kernels.cuh"

namespace q3t {

struct FrameArgs {
  const Phase *ph;  // device array of n phases
  int n;
  unsigned *bar;    // grid-barrier counter (zeroed by frame_launch before the kernel)
  int *err;         // bit 12 set with the wait bits when a bounded wait gave up
  int hc;           // hardware cluster size of the launch
  unsigned long long *trace;  // nullable: [grid][n][8] globaltimer ns per CTA and phase: start; GEMM
                              // (last round): X staged, weights landed, MMAs done, first cluster
                              // barrier passed, epilogue done, second cluster barrier passed; done
};

// Resident grid and cluster size of k_frame on `device` (false: it cannot
// run there, e.g. too few SMs can host clusters).
bool frame_init(int device, int *grid, int *hc);
// Whether k_frame can run this phase with hardware clusters of hc CTAs.
bool frame_phase_ok(const Phase &p, int hc);
// Zeroes the barrier counter and launches k_frame on `st`.
void frame_launch(const FrameArgs &a, int grid, cudaStream_t st);

}  // namespace q3t
