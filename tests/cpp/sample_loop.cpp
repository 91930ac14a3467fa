// The decode loop's use of the drop-in sample_token (ane_lm::cuda,
// core/cuda_ops.h), as ANE-LM's generate.cpp:80-129 calls the reference's:
// srand48(seed) once, then `steps` calls on device logits, each appending
// its token to the host history.  Writes the tokens and the device's free
// memory after the first call and after the last one to argv[2]; reads the
// logits rows, the parameters and the initial history from argv[1].
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "cuda_ops.h"

namespace cu = ane_lm::cuda;

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* in = fopen(argv[1], "rb");
    FILE* out = fopen(argv[2], "wb");
    if (!in || !out) return 2;
    int hdr[6];  // nrows, vocab, ctx, hist0_len, steps, seed
    float par[3];  // temperature, repetition penalty, frequency penalty
    if (fread(hdr, sizeof(int), 6, in) != 6 || fread(par, sizeof(float), 3, in) != 3) return 2;
    const int nrows = hdr[0], vocab = hdr[1], steps = hdr[4];
    std::vector<float> logits((size_t)nrows * vocab);
    std::vector<int> recent((size_t)hdr[3]);
    if (fread(logits.data(), sizeof(float), logits.size(), in) != logits.size()) return 2;
    if (fread(recent.data(), sizeof(int), recent.size(), in) != recent.size()) return 2;
    float* dl = nullptr;
    if (cudaMalloc(&dl, logits.size() * sizeof(float)) != cudaSuccess) return 3;
    cudaMemcpy(dl, logits.data(), logits.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaStream_t s;
    cudaStreamCreate(&s);
    cu::set_stream(s);
    cu::SamplingParams p;
    p.temperature = par[0];
    p.repetition_penalty = par[1];
    p.repetition_context_size = hdr[2];
    p.frequency_penalty = par[2];
    srand48(hdr[5]);
    std::vector<int> toks;
    size_t free_first = 0, free_last = 0, total = 0;
    for (int i = 0; i < steps; i++) {
        const int t = cu::sample_token(dl + (size_t)(i % nrows) * vocab, vocab, p, recent);
        if (t < 0) return 4;
        toks.push_back(t);
        recent.push_back(t);
        if (i == 0) cudaMemGetInfo(&free_first, &total);
    }
    cudaMemGetInfo(&free_last, &total);
    fwrite(toks.data(), sizeof(int), toks.size(), out);
    const long long mem[2] = {(long long)free_first, (long long)free_last};
    fwrite(mem, sizeof(mem), 1, out);
    fclose(out);
    return 0;
}
