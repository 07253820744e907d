// Evaluates cuRAND's Philox4x32-10 block function (curand_philox4x32_x.h)
// on a list of (key, counter) inputs read from stdin, one per line:
//   key0 key1 c0 c1 c2 c3      (decimal u32)
// and prints the four output words per line. Used only to generate
// tests/golden/philox_kat.json, the cross-implementation pin of the oracle's
// Philox (crates/ops/src/rng.rs:43-60).
#include <cstdio>
#include <vector>

#include <curand_kernel.h>

__global__ void blocks(const uint4 *ctr, const uint2 *key, uint4 *out, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = curand_Philox4x32_10(ctr[i], key[i]);
}

int main() {
    std::vector<uint4> c;
    std::vector<uint2> k;
    unsigned a, b, x, y, z, w;
    while (scanf("%u %u %u %u %u %u", &a, &b, &x, &y, &z, &w) == 6) {
        k.push_back(make_uint2(a, b));
        c.push_back(make_uint4(x, y, z, w));
    }
    int n = (int)c.size();
    uint4 *dc, *dout;
    uint2 *dk;
    if (cudaMalloc(&dc, n * sizeof(uint4)) || cudaMalloc(&dk, n * sizeof(uint2)) ||
        cudaMalloc(&dout, n * sizeof(uint4)))
        return 1;
    cudaMemcpy(dc, c.data(), n * sizeof(uint4), cudaMemcpyHostToDevice);
    cudaMemcpy(dk, k.data(), n * sizeof(uint2), cudaMemcpyHostToDevice);
    blocks<<<(n + 127) / 128, 128>>>(dc, dk, dout, n);
    std::vector<uint4> out(n);
    if (cudaMemcpy(out.data(), dout, n * sizeof(uint4), cudaMemcpyDeviceToHost) != cudaSuccess)
        return 2;
    for (int i = 0; i < n; ++i) printf("%u %u %u %u\n", out[i].x, out[i].y, out[i].z, out[i].w);
    return 0;
}
