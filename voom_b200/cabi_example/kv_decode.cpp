// C-ABI example and profiling driver: plans, uploads and decodes a directory of
// zstd frames (src.bin, jobs.bin as voom_zstd_job records, raw.bin = expected
// output) with voom_zstd_plan_create / voom_zstd_decode, three times, then
// checks every status word and the bytes.  No Python: ncu can attach to it.
// Inputs: any host script that writes the compressed bytes, the job records
// (voom_b200.formats.packed.body_job gives a vpack body's interleaved job) and
// the expected output image with the jobs' outputs packed end to end.
//   nvcc -O2 -std=c++17 -I include -o voom_b200/cabi_example/kv_decode \
//        voom_b200/cabi_example/kv_decode.cpp -L voom_b200 -lvoom_b200 \
//        -Xlinker -rpath -Xlinker '$ORIGIN/..'
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include <cuda_runtime.h>
#include "voom_b200.h"
static std::vector<uint8_t> rd(const char* p) {
  FILE* f = fopen(p, "rb"); if (!f) { perror(p); exit(1); }
  fseek(f, 0, SEEK_END); long n = ftell(f); fseek(f, 0, SEEK_SET);
  std::vector<uint8_t> v(n); if (fread(v.data(), 1, n, f) != size_t(n)) exit(1); fclose(f); return v;
}
int main(int argc, char** argv) {
  if (argc < 2) { fprintf(stderr, "usage: kv_decode DIR\n"); return 2; }
  const std::string dir = argv[1];
  auto src = rd((dir + "/src.bin").c_str()), jb = rd((dir + "/jobs.bin").c_str()), raw = rd((dir + "/raw.bin").c_str());
  const uint32_t nj = uint32_t(jb.size() / sizeof(voom_zstd_job));
  const voom_zstd_job* jobs = reinterpret_cast<const voom_zstd_job*>(jb.data());
  void* plan = voom_zstd_plan_create(src.data(), src.size(), jobs, nj, 0);
  voom_zstd_plan_info info; voom_zstd_plan_info_get(plan, &info);
  std::vector<uint8_t> img(info.plan_bytes); voom_zstd_plan_image(plan, img.data(), img.size());
  uint8_t *d_src, *d_img, *d_scr, *d_out; uint32_t* d_st;
  cudaMalloc(&d_src, src.size() + 16); cudaMalloc(&d_img, img.size()); cudaMalloc(&d_scr, info.scratch_bytes);
  cudaMalloc(&d_out, raw.size()); cudaMalloc(&d_st, 4 * nj);
  cudaMemcpy(d_src, src.data(), src.size(), cudaMemcpyHostToDevice); cudaMemset(d_src + src.size(), 0, 16);
  cudaMemcpy(d_img, img.data(), img.size(), cudaMemcpyHostToDevice);
  for (int r = 0; r < 3; r++) {
    cudaMemset(d_st, 0, 4 * nj);
    int rc = voom_zstd_decode(d_src, d_img, plan, d_scr, d_out, d_st, nullptr);
    if (rc) { printf("decode rc %d\n", rc); return 1; }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) { printf("cuda error\n"); return 1; }
  std::vector<uint8_t> out(raw.size()); std::vector<uint32_t> st(nj);
  cudaMemcpy(out.data(), d_out, out.size(), cudaMemcpyDeviceToHost);
  cudaMemcpy(st.data(), d_st, 4 * nj, cudaMemcpyDeviceToHost);
  for (uint32_t j = 0; j < nj; j++) if (st[j]) { printf("status %u at %u\n", st[j], j); return 1; }
  if (memcmp(out.data(), raw.data(), raw.size())) { printf("mismatch\n"); return 1; }
  printf("ok %u jobs, %zu bytes, direct %u\n", nj, raw.size(), info.n_direct_jobs);
  voom_zstd_plan_destroy(plan);
  return 0;
}
