// Deterministic reduction of per-sequence partial rows over the sequence axis.
//
// rows (S, K) -> out (K), in two fixed-order stages so the result is bitwise
// reproducible: stage 1 sums kRowsPerGroup consecutive rows per column (one CTA column
// block x row group), stage 2 sums the groups in order and scatters the K columns into up
// to kMaxSegments output arrays (consecutive column ranges; NULL arrays are skipped).
#pragma once

#include "semx_common.cuh"

namespace semx {
namespace {

constexpr int kRowsPerGroup = 32;
constexpr int kMaxSegments = 8;

struct Segments {
  float* out[kMaxSegments];
  int64_t len[kMaxSegments];
  int n;
};

__global__ void colsum_stage1(const float* __restrict__ rows, int64_t S, int64_t K,
                              float* __restrict__ group_sums) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  const int64_t r0 = (int64_t)blockIdx.y * kRowsPerGroup;
  const int64_t r1 = min(r0 + kRowsPerGroup, S);
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) acc += rows[r * K + k];
  group_sums[(int64_t)blockIdx.y * K + k] = acc;
}

__global__ void colsum_stage2(const float* __restrict__ group_sums, int64_t G, int64_t K,
                              Segments seg) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  int64_t off = k;
  int which = 0;
  while (which < seg.n && off >= seg.len[which]) {
    off -= seg.len[which];
    ++which;
  }
  if (which >= seg.n || seg.out[which] == nullptr) return;
  float acc = 0.f;
  for (int64_t q = 0; q < G; ++q) acc += group_sums[q * K + k];
  seg.out[which][off] = acc;
}

inline size_t colsum_group_floats(int64_t S, int64_t K) {
  return (size_t)cdiv(S, kRowsPerGroup) * (size_t)K;
}

// rows: (S, K); group_sums: colsum_group_floats(S, K) floats of scratch.
inline int colsum(const float* rows, int64_t S, int64_t K, float* group_sums, const Segments& seg,
                  cudaStream_t st) {
  if (K <= 0) return SEMX_OK;
  const int64_t G = cdiv(S, kRowsPerGroup);
  if (G > 0) {
    colsum_stage1<<<dim3((unsigned)cdiv(K, 256), (unsigned)G), 256, 0, st>>>(rows, S, K, group_sums);
    int rc = check_launch("colsum_stage1");
    if (rc != SEMX_OK) return rc;
  }
  colsum_stage2<<<(unsigned)cdiv(K, 256), 256, 0, st>>>(group_sums, G, K, seg);
  return check_launch("colsum_stage2");
}

}  // namespace
}  // namespace semx
