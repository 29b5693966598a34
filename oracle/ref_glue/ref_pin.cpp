// ref_pin.cpp -- C entry points over the reference's own host decode helpers.
//
// TEST INFRASTRUCTURE ONLY.  This file holds no algorithm: it #includes the
// reference header orders/F1-ref/exl3_dequant.cuh where it lies in the
// reference tree (the include path is given by oracle/build_oracle.py) and
// exports its functions with a C ABI, so the Python tests can compare the
// oracle against the reference compiled from source.  Output goes to
// oracle/_ref/ only.
#include <cstddef>
#include <cstdint>

#include "exl3_dequant.cuh"

extern "C" {

uint16_t ref_read_window(const uint16_t* packed, size_t words, size_t bit) {
    return vllm_exl3::read_window(packed, words, bit);
}

uint16_t ref_decode_codebook_bits(uint16_t window, int cb) {
    return vllm_exl3::decode_codebook_bits(window, cb);
}

float ref_decode_mcg(uint16_t window) { return vllm_exl3::decode_mcg(window); }

float ref_decode_mul1(uint16_t window) { return vllm_exl3::decode_mul1(window); }

float ref_decode_weight(const uint16_t* packed, size_t words, int index, int bits, int mcg) {
    return vllm_exl3::decode_weight(packed, words, index, bits, mcg != 0);
}

void ref_hadamard(float* values, int n) { vllm_exl3::hadamard(values, n); }

float ref_half_bits_to_float(uint16_t bits) { return vllm_exl3::half_bits_to_float(bits); }

}
