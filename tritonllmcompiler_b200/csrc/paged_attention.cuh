// Launch parameters and split plan shared by the paged decode entry points.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace tllm {
namespace paged {

struct Params {
  const void *q;
  const void *k_cache;
  const void *v_cache;
  const int32_t *block_tables;
  const int32_t *context_lens;
  void *o;
  float *ws_ml;   // [B, H, num_splits, 2] (running max in log2 units, sum of exponentials)
  float *ws_acc;  // [B, H, num_splits, D] unnormalised P*V partials
  int64_t B, H, D;
  int64_t num_blocks;
  int block_size, log2_bs;
  int max_tokens;  // max_blocks * block_size: tokens past this are never read
  int chunk;       // tokens per split
  int num_splits;
  int64_t sq0, sq1, sq3;
  int64_t skc0, skc1, skc2, skc3;
  int64_t svc0, svc1, svc2, svc3;
  int64_t sbt0, sbt1;
  int64_t so0, so1, so3;
  float sm_scale;
  // Grouped-query decode (run_gqa): query heads per KV head and the number of KV heads; the
  // caches' head index is the KV head, q / o / the workspace use the H = G * Hkv query heads.
  int G = 1;
  int64_t Hkv = 0;
  // Sq new tokens per sequence (q [B, H, Sq, D] with token stride sq2, o likewise with so2);
  // with causal set, new token s sits at position len - Sq + s and sees the keys up to it.
  // The workspace and the merge then index rows (b, h, s). The single-token entries keep 1.
  int Sq = 1;
  int causal = 0;
  int64_t sq2 = 0, so2 = 0;
};

struct Plan {
  int64_t max_tokens = 0;
  int64_t chunk = 512;
  int64_t num_splits = 1;
  size_t ws_ml_floats = 0;
  size_t ws_acc_floats = 0;
  size_t ws_acc_offset = 0;
  size_t ws_bytes = 0;
};

// Split plan for a problem: chunk length and number of splits depend only on the shape
// and the SM count, so the workspace size can be queried before the launch.
Plan plan(int64_t B, int64_t H, int64_t D, int64_t block_size, int64_t max_blocks, int sms);
// Shape/stride/alignment checks shared by every entry point (sets the last error).
int validate(const Params &p);
// Reads and clears this file's device error word.
int read_status(int *out);
// Enqueues the split kernel (and the merge kernel when num_splits > 1).
int run(const Params &p, int dtype, cudaStream_t st);
// Enqueues the merge of the split partials into o for the p.H heads.
int run_merge(const Params &p, int dtype, cudaStream_t st);

// Decode of Sq new tokens with G = H / Hkv query heads per KV head, G * Sq <= 16 query rows
// per KV head: each token's K and V rows are read once for all rows. The plan is made over
// the KV heads; its workspace holds the partials of all H * Sq query rows.
Plan plan_gqa(int64_t B, int64_t H, int64_t Hkv, int64_t Sq, int64_t D, int64_t block_size,
              int64_t max_blocks, int sms);
// Whether run_gqa handles this group size, token count, head dim and plan (otherwise use
// another path).
bool gqa_supported(int64_t G, int64_t Sq, int64_t D, const Plan &pl);
int run_gqa(const Params &p, int dtype, cudaStream_t st);

}  // namespace paged
}  // namespace tllm
