// aipu_dequant_dump -- exact dequantisation of raw GGUF blocks on the GPU through the library's C ABI.
//
//   usage: aipu_dequant_dump <q4_k|q6_k|q8_0|f16> <raw_blocks.bin> <out_f32.bin>
//
// Same command line and file formats as the reference's ggml dump tool (tools/dequant_dump.c:1-39): the
// input is N whole blocks (Q4_K 144 B and Q6_K 210 B per 256 weights, Q8_0 34 B per 32 weights; F16
// 2 B per weight), the output is the fp32 weights in order. The blocks are dequantised by
// aipu_q4k_dequant (bit-identical to tools/q4k_ref.py and so to ggml's dequantize_row_*), so this
// binary can stand in for the reference's dump in its GGUF cross-check (tools/gguf_crosscheck.py:69-117)
// wherever GGUF files exist. Exit codes: 0 ok, 1 I/O or CUDA error, 2 usage.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "aipu_q4k.h"

namespace {

struct Kind {
  const char* name;
  int wtype;
  long block_bytes;
  long block_weights;
};

const Kind kKinds[] = {{"q4_k", AIPU_Q4_K, 144, 256},
                       {"q6_k", AIPU_Q6_K, 210, 256},
                       {"q8_0", AIPU_Q8_0, 34, 32},
                       {"f16", AIPU_F16, 2, 1}};

int fail_cuda(cudaError_t e, const char* what) {
  std::fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  return 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 4) {
    std::fprintf(stderr, "usage: %s <q4_k|q6_k|q8_0|f16> <in> <out>\n", argc > 0 ? argv[0] : "aipu_dequant_dump");
    return 2;
  }
  const Kind* kind = nullptr;
  for (const Kind& k : kKinds)
    if (std::strcmp(argv[1], k.name) == 0) kind = &k;
  if (!kind) {
    std::fprintf(stderr, "unknown type %s (q4_k, q6_k, q8_0 or f16)\n", argv[1]);
    return 2;
  }
  FILE* fi = std::fopen(argv[2], "rb");
  if (!fi) {
    std::perror(argv[2]);
    return 1;
  }
  std::fseek(fi, 0, SEEK_END);
  const long size = std::ftell(fi);
  std::fseek(fi, 0, SEEK_SET);
  if (size <= 0 || size % kind->block_bytes) {
    std::fprintf(stderr, "size %ld is not a positive multiple of the %s block (%ld bytes)\n", size, kind->name,
                 kind->block_bytes);
    std::fclose(fi);
    return 1;
  }
  const long nblocks = size / kind->block_bytes;
  const long nweights = nblocks * kind->block_weights;
  // whole 16-byte chunks: the kernels may read up to the next 16-byte boundary
  std::vector<unsigned char> raw(static_cast<size_t>((size + 15) / 16 * 16), 0);
  if (std::fread(raw.data(), 1, static_cast<size_t>(size), fi) != static_cast<size_t>(size)) {
    std::perror("read");
    std::fclose(fi);
    return 1;
  }
  std::fclose(fi);

  void* d_in = nullptr;
  float* d_out = nullptr;
  cudaError_t e = cudaMalloc(&d_in, raw.size());
  if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc");
  e = cudaMalloc(reinterpret_cast<void**>(&d_out), sizeof(float) * static_cast<size_t>(nweights));
  if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc");
  e = cudaMemcpy(d_in, raw.data(), raw.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemcpy");
  // one row of all the weights (the row layout is a concatenation of blocks along K)
  int rc = aipu_q4k_dequant(kind->wtype, d_in, 1, nweights, d_out, AIPU_DT_F32, nullptr);
  if (rc != AIPU_OK) {
    std::fprintf(stderr, "aipu_q4k_dequant: %d (%s)\n", rc, aipu_last_error());
    return 1;
  }
  std::vector<float> out(static_cast<size_t>(nweights));
  e = cudaMemcpy(out.data(), d_out, sizeof(float) * out.size(), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMemcpy");
  cudaFree(d_in);
  cudaFree(d_out);
  FILE* fo = std::fopen(argv[3], "wb");
  if (!fo) {
    std::perror(argv[3]);
    return 1;
  }
  const size_t wrote = std::fwrite(out.data(), sizeof(float), out.size(), fo);
  std::fclose(fo);
  if (wrote != out.size()) {
    std::perror("write");
    return 1;
  }
  std::fprintf(stderr, "dequantized %ld blocks (%ld weights) as %s\n", nblocks, nweights, kind->name);
  return 0;
}
