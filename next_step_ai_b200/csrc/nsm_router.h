// nsm_router.h -- router kernel parameters and launchers (nsm_router.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "nsm_internal.h"

namespace nsm {

struct RouterAParams {
  const void* x;
  int x_dtype;
  float* residual;
  const void* y_prev;
  int y_prev_dtype;
  const void* norm_w;
  int norm_w_dtype;
  float eps;
  int use_norm;
  const void* enc_w;  // may be null: x preparation only
  const void* enc_b;
  int wdtype;
  int rank;
  int basis_top_k;
  int H;
  int cols_per_cta;  // set by router_a_launch
  // y_prev = the previous layer's down partials pending in ws (summed here,
  // across ranks through `ex` when ex.world > 1)
  int pending;
  ExchangeDev ex;
  // 1: the scores kernel that follows reduces the partial latents (no last-CTA
  // reduction here); 0: the last CTA reduces them (x-prep-only launches)
  int reduce_in_scores;
  int multi_rows;  // > 0: routing only for rows = gridDim.y (row r reads x + r*H; per-row partials; no x16)
  DecodeWs ws;
};

struct RouterBParams {
  const void* score_w;
  const void* score_b;
  int wdtype;
  const float* dbn;
  int legacy;
  int rank;
  int NB;
  int top_k;
  int32_t* idx_out;
  float* score_out;
  float* latent_out;
  const int32_t* slot_of_block;
  int block_begin;
  int block_end;
  int pool_rows;
  // reduction of the router kernel's partials, done by every scores CTA
  int reduce_latent;
  int nparts;         // router kernel CTAs
  int use_norm;
  float eps;
  int H;
  const void* enc_b;
  int basis_top_k;
  uint32_t* epoch_counter;  // exchange epoch to advance (NULL without an exchange)
  int multi_rows;           // > 0: routing only, one row per grid y (scores) / per CTA (top-k)
  DecodeWs ws;
};
// CTAs of the router kernel for hidden size H (kRouterMaxCtas at most).
int router_a_ctas(int H, int* cols_per_cta);

int router_setup();
int router_a_launch(const RouterAParams& a, cudaStream_t stream);
// Scores kernel, then (topk) the top-k kernel.
int router_b_launch(const RouterBParams& b, cudaStream_t stream, bool topk = true);
// Routing only for `rows` rows of x (row-major [rows][H]) into idx_out [rows][k].
int router_rows_launch(const RouterAParams& a, RouterBParams b, int rows, cudaStream_t stream);
int select_given_launch(const RouterBParams& b, const int32_t* idx_in, int k, cudaStream_t stream);

}  // namespace nsm
