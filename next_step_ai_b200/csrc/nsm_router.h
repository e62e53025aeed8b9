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
  DecodeWs ws;
};

int router_setup();
int router_a_launch(const RouterAParams& a, cudaStream_t stream);
int router_b_launch(const RouterBParams& b, cudaStream_t stream);
int select_given_launch(const RouterBParams& b, const int32_t* idx_in, int k, cudaStream_t stream);

}  // namespace nsm
