// Exercises the reference-signature C++ layer (ane-lm_b200/core/cuda_ops.h)
// the way ANE-LM's own code would call it, on device buffers.  Reads inputs
// from argv[1] and writes every result to argv[2] (raw little-endian arrays,
// in the order below); tests/test_gpu_cpp_layer.py compares them with the
// oracle.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "cuda_ops.h"

namespace cu = ane_lm::cuda;

template <typename T>
static T* to_dev(const std::vector<T>& h) {
    T* d = nullptr;
    cudaMalloc(&d, h.size() * sizeof(T));
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}
template <typename T>
static std::vector<T> to_host(const T* d, size_t n) {
    std::vector<T> h(n);
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}
template <typename T>
static void put(FILE* f, const std::vector<T>& v) { fwrite(v.data(), sizeof(T), v.size(), f); }
template <typename T>
static std::vector<T> get(FILE* f, size_t n) {
    std::vector<T> v(n);
    if (fread(v.data(), sizeof(T), n, f) != n) { fprintf(stderr, "short input\n"); exit(2); }
    return v;
}

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* in = fopen(argv[1], "rb");
    FILE* out = fopen(argv[2], "wb");
    if (!in || !out) return 2;
    const int dim = 2048, hd = 128, nq = 16, nkv = 8, n = 3072, vocab = 151936;
    auto x = get<float>(in, dim);
    auto w = get<float>(in, dim);
    auto qk = get<float>(in, (nq + nkv) * hd);
    auto cosr = get<float>(in, hd / 2);
    auto sinr = get<float>(in, hd / 2);
    auto g = get<float>(in, n);
    auto z = get<float>(in, n);
    auto logits = get<float>(in, vocab);
    auto hist = get<int>(in, 300);
    auto bf = get<uint16_t>(in, 1000);
    const int cap = 300, a_start = 250, a_len = 290;
    auto kc = get<float>(in, (size_t)cap * nkv * hd);
    auto vc = get<float>(in, (size_t)cap * nkv * hd);

    cudaStream_t s;
    cudaStreamCreate(&s);
    cu::set_stream(s);

    float* dx = to_dev(x);
    float* dw = to_dev(w);
    cu::rmsnorm(dx, dx, dw, dim, 1e-6f);  // in place, as models/llm/qwen3.cpp:530
    cudaStreamSynchronize(s);
    put(out, to_host(dx, dim));

    float* dq = to_dev(qk);
    float* dcos = to_dev(cosr);
    float* dsin = to_dev(sinr);
    cu::apply_rope_cached(dq, dq + nq * hd, nq, nkv, hd, hd, hd, hd, 777, 1e6f, dcos, dsin);
    cudaStreamSynchronize(s);
    put(out, to_host(dq, qk.size()));
    float* dq2 = to_dev(qk);
    cu::apply_rope_cached(dq2, dq2 + nq * hd, nq, nkv, hd, hd, hd, hd, 777, 1e6f, nullptr, nullptr);
    cudaStreamSynchronize(s);
    put(out, to_host(dq2, qk.size()));

    float* dg = to_dev(g);
    cu::silu_vec_inplace(dg, n, nullptr);
    cudaStreamSynchronize(s);
    put(out, to_host(dg, n));
    float* dy = to_dev(g);
    float* dz = to_dev(z);
    cu::mul_sigmoid_inplace(dy, dz, n, nullptr);
    cudaStreamSynchronize(s);
    put(out, to_host(dy, n));

    float* dl = to_dev(logits);
    float* dsm = to_dev(logits);
    cu::softmax(dsm, vocab);
    cudaStreamSynchronize(s);
    put(out, to_host(dsm, vocab));

    cu::SamplingParams sp;  // 0.6 / 1.2 / 256 / 0.1, core/sampling.h:7-12
    std::vector<int> recent(hist.begin(), hist.end());
    std::vector<int> toks;
    srand48(4242);
    for (int i = 0; i < 4; i++) toks.push_back(cu::sample_token(dl, vocab, sp, recent));
    cu::SamplingParams greedy;
    greedy.temperature = 0.0f;
    toks.push_back(cu::sample_token(dl, vocab, greedy, recent));
    toks.push_back(cu::sample_token(dl, vocab, sp, {}));
    put(out, toks);

    uint16_t* db = to_dev(bf);
    uint16_t* dh = nullptr;
    cudaMalloc(&dh, bf.size() * 2);
    cu::bf16_to_f16_vec(dh, db, (int)bf.size());
    cudaStreamSynchronize(s);
    put(out, to_host(dh, bf.size()));

    // hybrid-model row ops, one head per call as models/llm/qwen3_5.cpp:528-550
    float* dgx = to_dev(x);
    float* dgz = to_dev(z);
    float* dgo = nullptr;
    cudaMalloc(&dgo, dim * sizeof(float));
    for (int h = 0; h < dim / hd; h++) cu::rmsnorm_gated(dgo + h * hd, dgx + h * hd, dgz + h * hd, dw, hd);
    cudaStreamSynchronize(s);
    put(out, to_host(dgo, dim));
    float* dl2 = to_dev(qk);
    for (int h = 0; h < nq + nkv; h++) cu::l2_normalize(dl2 + h * hd, hd);
    cudaStreamSynchronize(s);
    put(out, to_host(dl2, qk.size()));

    // gqa_attention over a wrapped ring (core/cpu_ops.cpp:173-240)
    float* dkc = to_dev(kc);
    float* dvc = to_dev(vc);
    float* dqa = to_dev(qk);
    float* dao = nullptr;
    cudaMalloc(&dao, nq * hd * sizeof(float));
    cu::gqa_attention(dao, dqa, dkc, dvc, nq, nkv, hd, hd, a_start, a_len, cap);
    cudaStreamSynchronize(s);
    put(out, to_host(dao, (size_t)nq * hd));
    cu::gqa_attention(dao, dqa, dkc, dvc, nq, nkv, hd, hd, 7, 0, cap);  // empty cache -> zeros
    cudaStreamSynchronize(s);
    put(out, to_host(dao, (size_t)nq * hd));

    // KV ring bookkeeping: 7 appends into a ring of 4
    std::vector<int> ring;
    int rs = 0, rl = 0;
    for (int i = 0; i < 7; i++) ring.push_back(cu::kv_ring_advance(&rs, &rl, 4));
    ring.push_back(rs);
    ring.push_back(rl);
    put(out, ring);

    // a failing call: reported through last_status, the process continues
    cu::rmsnorm(dx, dx, nullptr, dim, 1e-6f);
    std::vector<int> st = {cu::last_status()};
    put(out, st);
    fclose(out);
    return 0;
}
