/* Minimal stand-in for ggml.h, used ONLY to compile parakeet.cpp's own CPU
 * mel front end (src/mel.cpp, src/fft.cpp, src/pos_enc.cpp) into oracle/_ref.
 * Those files use nothing from ggml but the tensor struct's shape field and an
 * opaque data pointer; this header declares exactly that (test infrastructure,
 * not product code). */
#pragma once
#include <stddef.h>
#include <stdint.h>

struct ggml_tensor {
  int type;
  int64_t ne[4];
  void* data;
};
