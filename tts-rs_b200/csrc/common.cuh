// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define Q3T_DEV __device__ __forceinline__

namespace q3t {

using bf16 = __nv_bfloat16;

Q3T_DEV float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
Q3T_DEV uint16_t f2bf(float f) {
  bf16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&h);
}
Q3T_DEV uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
Q3T_DEV float bf16_round(float f) { return bf2f(f2bf(f)); }

// Programmatic dependent launch: everything before pdl_wait() may only read
// data no earlier kernel writes (weights, and the metadata and page tables
// that host copies put in place before the launch); pdl_wait() returns once the
// preceding grid has completed and its memory is visible.  Both are no-ops
// when the kernel was launched without the PDL attribute.
Q3T_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
Q3T_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
Q3T_DEV uint4 ldg_stream(const uint4 *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// D = A * B + D, m16n8k16, bf16 inputs, f32 accumulators.
Q3T_DEV void mma_16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

Q3T_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
Q3T_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024 (uses 33 floats of smem).
Q3T_DEV float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}

Q3T_DEV float silu(float x) { return x / (1.f + expf(-x)); }

Q3T_DEV uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---- asynchronous global -> shared copies (16 bytes; src_bytes < 16 zero-fills the rest) ----
Q3T_DEV void cp_async16(void *smem, const void *gmem, int src_bytes) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
Q3T_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
Q3T_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Four 8x8 b16 matrices from shared memory, transposed (lanes 8i..8i+7 give
// the row addresses of matrix i; register i receives matrix i).
Q3T_DEV void ldmatrix_x4_trans(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_addr(p)));
}

// ---- thread-block clusters (distributed shared memory) ----

// 16-byte load from the shared memory of cluster CTA `rank` at the address
// that p has in this CTA.
Q3T_DEV float4 ld_cluster_f4(const float *p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(p)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// All threads of all CTAs of the cluster; shared-memory writes before it are
// visible to every CTA of the cluster after it.
Q3T_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace q3t
