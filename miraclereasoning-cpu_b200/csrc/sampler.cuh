// Seeded top-k / top-p sampling on the device (sampler.cu): the reference's
// procedure (model.py:343-352, NumPy's Generator) reproduced to the bit.
#pragma once

#include "common.cuh"

namespace mr {

struct Sampler;

struct SampleParams {
    double temperature, top_p;  // temperature 0: NumPy's argmax
    int top_k;                  // 0: every token
    int eos, max_new;           // stop after eos or max_new tokens
};

int sampler_create(int vocab, Sampler **out);
void sampler_destroy(Sampler *s);
// PCG64 state of numpy.random.default_rng(seed): state (high, low 64 bits), increment (high, low).
int sampler_seed(Sampler *s, cudaStream_t stream, const unsigned long long pcg[4]);
// Queues one token from `logits` (vocab floats on the device): its id goes to *token_slot
// (the next step's input) and to out[count]; stop_flag (optional) is set when the
// generation ends (EOS, max_new, a non-finite logit).  Does nothing once stopped.
int sampler_step(Sampler *s, cudaStream_t stream, const float *logits, const SampleParams &p, int *token_slot,
                 int *out, int *stop_flag);
// Tokens produced so far and whether a non-finite logit stopped the generation (synchronous).
int sampler_result(Sampler *s, cudaStream_t stream, int *count, int *nonfinite);

}  // namespace mr
