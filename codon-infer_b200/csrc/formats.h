// Host-side codon-infer formats: presets, CODQ header, tensor layouts, quantizers, tokenizer.
#pragma once

#include <cstdint>
#include <functional>
#include <string>

#include "../../include/esm_b200.h"

namespace esm {

// CodqHeader, src/lib.rs:887-897: 64 bytes, little-endian, repr(C).
struct CodqHeader {
  char magic[4];
  uint32_t version;
  uint32_t dtype;
  uint32_t arch;
  uint32_t n_layers;
  uint32_t dim;
  uint32_t hidden_dim;
  uint32_t vocab_size;
  uint8_t reserved[32];
  // Empty string when the header is coherent (with cfg when given, else with its own arch).
  std::string validate(const esm_config* cfg) const;
};
static_assert(sizeof(CodqHeader) == 64, "CODQ header is 64 bytes");

bool config_preset(int arch, esm_config* out);
bool detect_from_file_len(uint64_t len, esm_config* out);
int64_t lm_head_floats(const esm_config& c);
int64_t grouped_canonical_floats(const esm_config& c);
int64_t sequential_hf_floats(const esm_config& c);
int64_t matrix_bytes(int dtype, int64_t elems);
// Byte sizes of tensors 0..18 in EsmWeights order for `dtype`; entry 19 (classifier) is set to 0.
void tensor_layout(const esm_config& c, int dtype, int64_t out_bytes[ESM_NUM_TENSORS]);

void quantize_q8(const float* src, int64_t n, uint8_t* dst);
void quantize_q4(const float* src, int64_t n, uint8_t* dst);
void quantize_q3(const float* src, int64_t n, uint8_t* dst);  // BlockQ3_LUT, 14 bytes per 32 values
uint16_t q3_scale_to_half(float v);                            // f32_to_f16 of the reference
float q3_half_to_scale(uint16_t h);                            // f16_to_f32 of the reference
// Storage type of tensor `tensor` (EsmWeights order) in a model of type `model_dtype`.
int matrix_dtype(int model_dtype, int tensor);
int tokenize(const char* seq, int32_t* out, int32_t cap, int32_t* n_out);

}  // namespace esm
