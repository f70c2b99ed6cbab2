// Temperature sampling as a Gumbel-max argmax, so that it fuses into the
// lm_head epilogue that already reduces each row to its best column.
//
// The reference samples token ~ softmax(logits / T) with torch.multinomial
// (llm.py:215-219, llm_tp.py:609-616; logits / T rounds to bf16 there).
// argmax_v (bf16(logit_v / T) + G_v), with G_v i.i.d. standard Gumbel, is a
// draw from exactly that distribution (the Gumbel-max trick), needs no
// normalisation pass over the vocabulary, and splits over vocab shards: each
// tensor-parallel rank perturbs its own columns and the (score, id) argmax
// merge picks the global sample.
//
// Noise is counter-based, so a decode step can be replayed from a CUDA graph
// and every TP rank draws the same value for the same (row, vocab id):
//   key   = splitmix64(seed ^ splitmix64(counter))           once per row and step
//   h     = fmix32(fmix32(k_lo ^ (v * 0x9E3779B9)) + k_hi)   per vocab id v
//   u     = ((h >> 8) + 0.5) / 2^24  in (0, 1)
//   G     = -log(-log(u))
// splitmix64 is the SplitMix64 output function (Steele, Lea and Flood,
// OOPSLA 2014, as published by Vigna); fmix32 is the 32-bit finaliser of
// Appleby's MurmurHash3.  `counter` is the position of the token whose logits
// are sampled, which advances by one every decode step on the device.
#pragma once

#include <stdint.h>

namespace aacc {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint32_t fmix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

__host__ __device__ __forceinline__ uint64_t sample_key(int64_t seed, int64_t counter) {
  return splitmix64((uint64_t)seed ^ splitmix64((uint64_t)counter));
}

// Standard Gumbel noise for vocab id v under `key`.
__device__ __forceinline__ float gumbel_noise(uint64_t key, uint32_t v) {
  const uint32_t h = fmix32(fmix32((uint32_t)key ^ (v * 0x9E3779B9u)) + (uint32_t)(key >> 32));
  const float u = ((float)(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

}  // namespace aacc
