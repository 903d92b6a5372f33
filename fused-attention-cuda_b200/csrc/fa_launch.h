// fa_launch.h -- internal interface between the C-ABI layer (dispatch.cu) and the sm_100a
// kernel translation unit (fa_fwd_sm100.cu).  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "fa_sm100.h"

namespace fa_sm100 {

struct LaunchArgs {
  int dtype;  // FA_DTYPE_*
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int B, H, Hkv, N, D;
  float scale;
  bool causal;
  int block_n;  // keys per tile: 32, 64 or 128
  unsigned long long timeout_ns;
  int skip_kv_tile;  // fault injection, -1 = off
  void* workspace;   // fp32 only: tf32-rounded q|k|v, workspace_bytes_f32() bytes
  // Element strides of the (b, h, n) dimensions of q, k, v, o; d is contiguous.
  long long sq[3], sk[3], sv[3], so[3];
};

// Which key-tile widths this build instantiates for (dtype, D).
bool block_n_supported(int dtype, int D, int block_n);
int default_block_n(int dtype, int D, int N, int causal);

// Workspace of the fp32 path: tf32-rounded copies of q, k and v.
size_t workspace_bytes_f32(int B, int H, int Hkv, int N, int D);

// The checks fa_forward / fa_forward_strided make before launching (st may be null; the
// workspace is checked only when need_workspace): cudaSuccess, cudaErrorInvalidValue or
// cudaErrorNotSupported, exactly as those entry points would return them.
cudaError_t check_forward_args(int impl, int dtype, const void* q, const void* k, const void* v,
                               const void* o, const float* lse, const void* workspace,
                               bool need_workspace, const fa_params_t* p, const fa_strides_t* st);

// Validated arguments only; returns the launch status (never synchronises).
cudaError_t launch_forward(const LaunchArgs& a, cudaStream_t stream);

// Synchronises the current device, reads and clears the device status word.
cudaError_t read_and_clear_status(unsigned int* bits);

// Device-side status bits (which wait ran out).
enum StatusBits : unsigned int {
  kStQFull = 1u << 0,    // MMA warp waiting for the Q tile
  kStKFull = 1u << 1,    // MMA warp waiting for a K tile
  kStVFull = 1u << 2,    // MMA warp waiting for a V tile
  kStPFull = 1u << 3,    // MMA warp waiting for P from the softmax warps
  kStSFull = 1u << 4,    // softmax warps waiting for S
  kStODone = 1u << 5,    // softmax warps waiting for an O update
  kStKVEmpty = 1u << 6,  // producer waiting for a free K/V slot
  kStDrain = 1u << 7,    // exit path waiting for in-flight copies / MMAs
  kStSFree = 1u << 8,    // MMA warp waiting for the softmax warps to read S (lookahead kernel)
  kStPFree = 1u << 9,    // softmax warps waiting for a PV to release P (lookahead kernel)
  kStBounds = 1u << 10,  // FA_DEBUG_CHECKS builds: an index or address check failed
};

}  // namespace fa_sm100
