// Parameters shared by the two sparse-attention kernels (flash_mma.cu: mma.sync for head_dim < 128;
// flash_tc.cu: tcgen05/TMEM/TMA for head_dim 128).
#pragma once

#include "bb_common.cuh"

namespace bb {

constexpr float LOG2E = 1.4426950408889634f;

struct FlashParams {
  const void* q; int64_t sq_h, sq_t;
  const void* k; int64_t sk_h, sk_t;
  const void* v; int64_t sv_h, sv_t;
  const int32_t* idx; int64_t si_h, si_g, si_k;
  const uint8_t* mask; int64_t sm_b, sm_t;
  void* out; int64_t so_h, so_t;
  int64_t t, n, d, offset;
  int64_t num_heads, kv_groups;
  int64_t front, window;       // front already clipped to n
  int64_t route_k, route_groups, route_chunk;
  int64_t row_begin, row_end;
  float scale_log2;
  int splits;
  float* part_acc;             // [splits][BH][T][128] (split mode)
  float2* part_ml;             // [splits][BH][T]: (running max in log2 units, sum)
  int64_t bh;
  uint32_t serial;             // launch serial (cross-CTA abort of the tcgen05 kernels)
  // tcgen05 path: routed K/V rows gathered once per call, [bh][route_groups][route_kpad][128] each
  // (route_kpad = route_k rounded up to 128; empty slots are zero rows).
  void* kg;
  void* vg;
  int64_t route_kpad;
  int32_t* tile_min;           // [bh][route_groups][route_kpad / 128]: smallest routed position >= front
                               // (read as unsigned; all ones = none)
};

int flash_tc_launch(const bb_flash_args* a, FlashParams& p, cudaStream_t stream);
// Bytes of the tcgen05 path's gathered routed rows (K and V together; 0 without routes).
size_t flash_tc_gather_bytes(const bb_flash_args* a);
int flash_tc_splits(const bb_flash_args* a, int sms);
// Read and clear the current device's fault words (set by a kernel whose bounded wait gave up):
// one for the attention kernels, one for the tcgen05 routing kernels.
int flash_fault_take(int* code);
int routes_fault_take(int* code);
int decode_fault_take(int* code);
// Wait limit (ns) of the bounded waits of each unit's kernels, on the current device.
int flash_set_wait_limit(unsigned long long ns);
int routes_set_wait_limit(unsigned long long ns);
int decode_set_wait_limit(unsigned long long ns);
// Test hook of the attention kernels' abort path (see bb_debug_stall_attention).
int flash_set_stall(int on);

}  // namespace bb
