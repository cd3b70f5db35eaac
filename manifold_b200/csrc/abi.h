// Host helpers shared by the translation units of libgfn_b200.so.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/gfn_b200.h"

namespace gfn_abi {

// Records a printf-style message for gfn_last_error_message; returns status.
int fail(int status, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
int launch_status(const char* what);
bool aligned16(const void* p);

// The weight layout (K, KC) depends only on (d, H, r); the row blocking R
// also on the batch and the device.
struct Layout {
  int d, H, hd, r, NL, K, C, hpc, KC, nchunk, HS, CF, mix;
  long long LF;
  // training layout: head section + untransposed Wf (HST floats), forward and
  // transposed mixing chunks
  int HST;
  long long LFT;
};


int make_layout(int d, int H, int r, int NL, Layout* L);

// Device error words of the other translation units (see gfn_unit_error_word).
cudaError_t error_word_layered(int* v, int reset, cudaStream_t s);
cudaError_t error_word_probe(int* v, int reset, cudaStream_t s);
cudaError_t error_word_readout(int* v, int reset, cudaStream_t s);

}  // namespace gfn_abi
