// A decode loop written against the reference sampler's interface, run on
// the B200 sampler through qs_sampler_compat.h.
//
// It follows main.cu's chat() loop (main.cu:130-139): the prompt's tokens are
// fed for positions below the prompt length, the model's forward() gives the
// position's logits, and sample() runs at every position -- prefill included
// -- so the window and counts see every sampled token.  The transformer is a
// stub: forward() writes a bf16 row of logits to device memory from a hash
// of (token, position), standing in for the lm_head output of
// qwen_model.cuh:715-716 before its fp32 widening and host copy.
//
// qs_demo_decode is built into integration/libqs_decode_demo.so for the
// integration test, which replays the same logits through the reference's
// own sampler.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qs_sampler_compat.h"

namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352du;
    x ^= x >> 15; x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Stub forward(): logits[i] = bf16(scale * (u - 0.5)) with u from a hash of
// (token, pos, i); a few tokens per position get a raised logit so the
// distribution has a head like a language model's.
__global__ void stub_forward_kernel(__nv_bfloat16* out, int V, int token, int pos, uint32_t seed) {
    const uint32_t base = mix32(seed ^ mix32((uint32_t)token * 0x9E3779B9u ^ (uint32_t)pos * 0x85EBCA6Bu));
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        const uint32_t h = mix32(base ^ (uint32_t)i * 0xC2B2AE35u);
        float x = (float)(h >> 8) * (1.0f / 16777216.0f);  // [0, 1), exact
        x = (x - 0.5f) * 16.0f;
        if ((h & 1023u) == 7u) x += 12.0f;
        out[i] = __float2bfloat16_rn(x);
    }
}

}  // namespace

extern "C" {

// Runs n_steps positions of the loop; out_tokens[pos] is the token sampled
// at pos.  out_logits (host, n_steps x vocabulary bf16 bits, may be NULL)
// receives each position's logits.  device_logits = 1 samples the device
// row directly (sample_device), 0 copies it to the host as fp32 first
// (sample(), the reference's shape).  Returns 0, or -1 on a CUDA error.
__attribute__((visibility("default"))) int qs_demo_decode(
    int n_steps, const int* prompt, int n_prompt, float temperature, float topp, float minp, int top_k,
    float repetition_penalty, float frequency_penalty, float presence_penalty, int penalty_window,
    unsigned long long seed, int device_logits, int* out_tokens, uint16_t* out_logits) {
    const int V = QS_COMPAT_VOCAB;
    __nv_bfloat16* d_logits = nullptr;
    float* h_logits = nullptr;
    if (cudaMalloc(&d_logits, sizeof(__nv_bfloat16) * V) != cudaSuccess) return -1;
    if (cudaMallocHost(&h_logits, sizeof(float) * V) != cudaSuccess) { cudaFree(d_logits); return -1; }
    uint16_t* h_bits = reinterpret_cast<uint16_t*>(h_logits);  // staging for the bf16 row
    Sampler sampler;
    build_sampler(&sampler, temperature, topp, minp, top_k, repetition_penalty, frequency_penalty,
                  presence_penalty, penalty_window, seed);
    int rc = 0;
    int next = 0;
    for (int pos = 0; pos < n_steps && rc == 0; pos++) {
        const int token = pos < n_prompt ? prompt[pos] : next;
        stub_forward_kernel<<<148, 256>>>(d_logits, V, token, pos, (uint32_t)seed);
        if (cudaGetLastError() != cudaSuccess) { rc = -1; break; }
        if (out_logits) {
            if (cudaMemcpy(out_logits + (size_t)pos * V, d_logits, sizeof(uint16_t) * V,
                           cudaMemcpyDeviceToHost) != cudaSuccess) { rc = -1; break; }
        }
        if (device_logits) {
            next = sample_device(&sampler, d_logits, QS_BF16, nullptr);
        } else {
            // the reference's shape: fp32 logits on the host
            if (cudaMemcpy(h_bits, d_logits, sizeof(uint16_t) * V, cudaMemcpyDeviceToHost) != cudaSuccess) {
                rc = -1;
                break;
            }
            for (int i = V - 1; i >= 0; i--) {
                const uint32_t b = (uint32_t)h_bits[i] << 16;
                memcpy(&h_logits[i], &b, sizeof(float));
            }
            next = sample(&sampler, h_logits);
        }
        out_tokens[pos] = next;
    }
    free_sampler(&sampler);
    cudaFreeHost(h_logits);
    cudaFree(d_logits);
    return rc;
}

}  // extern "C"
