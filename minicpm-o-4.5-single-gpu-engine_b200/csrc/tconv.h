// Internal launch interface of the TF32 convolution kernel (tconv.cu; not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace t2w {

enum { TCONV_BIAS = 0, TCONV_SNAKE = 1, TCONV_RESID = 2, TCONV_ELU = 3, TCONV_LEAKY = 4 };

// out[row_mul m + row_add, n] (ldo floats per row) = epilogue(bias[n] + sum_tap sum_c A[m + tap_row0 + tap dil, c]
// W[n, tap Cp + c]) for m < M (M % 128 == 0), rows whose pad[row_mul m + row_add] != 0 zero (bias, snake, elu) or
// untouched (resid).  A fp32 [rows_a, lda] (rows outside [0, rows_a) read as zero), Cin % 4 == 0, W fp32 [N, taps Cp]
// with Cp = Cin rounded up to 32 (the columns past Cin of each tap zero), N a multiple of 128, or 64, or 32.  out2 with
// the bias or resid epilogue: Snake(out) (alpha / inv) into out2 as well.
//
// split_in (3xTF32, fp32-level accuracy; Cin % 32 == 0): A holds [hi | lo] (2 Cin floats per row: hi = a rounded to TF32, lo = a - hi
// rounded to TF32) and W per tap [W_hi | W_lo | W_hi] (3 Cin columns per tap), so the sum is
// hi W_hi + hi W_lo + lo W_hi.  split_out: the epilogue writes the output in that [hi | lo] form (2 N columns; not the
// residual update, whose stream stays plain); split_out2 the same for out2 (row stride ldo2, 0: ldo).
struct TConvArgs {
  const float* A = nullptr;
  int lda = 0, rows_a = 0;
  const float* W = nullptr;
  const float* bias = nullptr;
  int M = 0, N = 0, Cin = 0, taps = 1, tap_row0 = 0, dil = 1;
  float* out = nullptr;
  long long ldo = 0;
  int row_mul = 1, row_add = 0;
  const uint8_t* pad = nullptr;
  int epi = TCONV_BIAS;
  const float* alpha = nullptr;  // TCONV_SNAKE: this conv's Snake; with out2: the next Snake
  const float* inv = nullptr;
  float* out2 = nullptr;
  const float* resid_in = nullptr;  // TCONV_RESID: out = resid_in + bias + conv (padding rows copied), else out in place
  int split_in = 0, split_out = 0, split_out2 = 0;
  long long ldo2 = 0;
  float slope = 0.f;  // TCONV_LEAKY: the negative-side slope
  int* err = nullptr;
};
int launch_tconv(const TConvArgs& a, cudaStream_t st);

}  // namespace t2w
