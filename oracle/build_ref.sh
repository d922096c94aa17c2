#!/usr/bin/env bash
# Builds oracle/_ref/libpb_refpins.so: the reference's OWN CPU functions for
# this path, compiled from the reference sources where they lie. TEST
# INFRASTRUCTURE ONLY (it pins the oracle restatement; nothing ships it).
#
# No reference source is copied into this repository: each function is cut
# out of its file by line range at build time and piped straight into the
# compiler (stdin), followed by a few exported wrappers written here.
#
#   pq1_host.c:14-24, 78-121    pq1_h2f, pq1_split_repack, pq1_gemv_cpu (non-ternary)
#   fwd35_ref.c:42-43, 46-72    fbits/bitsf, f16f, ff16
#   fwd35_ref.c:333-344         Q8 / q8(): the Q8_0 activation quantizer
#   pq1_parity.c:13-23          mk_q8k: the parity gate's seeded Q8_K generator
#   pq1_parity.c:119-147        rms_ser / rms_ref: RMS + Q8_K quantizer chain
#   q8_gemv_cpu.c (whole file)  gemv_q8 / quant_row (main renamed away)
#   lfm3_nanode.cu:4598-4603    cpu_f2bf / cpu_bf2f
#   lfm3_nanode.cu:4658-4684    cpuchk_run's scalar leaf-order transcription
#   fwd8.c:312-317, 320-369     rms, YaRN rope table and rotation (8B constants)
#   fwd8.c:465-521              argmax, RS, frand01, sample_topkpp (libpb_sample.so)
#   pq1_host.c:373-434, 226     pq1_fa16_head (f16 flash-attention decode), silu tail
#
# Needs the reference checkout (default /root/reference, override with
# PB_REFERENCE_ROOT). Without it this script does nothing and exits 0.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
REF="${PB_REFERENCE_ROOT:-/root/reference}"
out="$here/_ref"
if [ ! -d "$REF/pulsar_arm" ]; then
  echo "build_ref: no reference tree at $REF; skipping"; exit 0
fi
CC=/usr/bin/gcc; [ -x "$CC" ] || CC=gcc
CXX=/usr/bin/g++; [ -x "$CXX" ] || CXX=g++
mkdir -p "$out"
B2="$REF/pulsar_arm/bonsai2"
CFL="-O2 -fPIC -ffp-contract=off -fopenmp -w"

# --- A: bonsai2 host functions (C) ------------------------------------------
{
  printf '#include <stdint.h>\n#include <string.h>\n#include <stdlib.h>\n#include <math.h>\n#include <stddef.h>\n'
  sed -n '14,24p'   "$B2/pq1_host.c"
  sed -n '78,121p'  "$B2/pq1_host.c"
  sed -n '42,43p'   "$B2/fwd35_ref.c"
  sed -n '46,72p'   "$B2/fwd35_ref.c"
  sed -n '333,344p' "$B2/fwd35_ref.c"
  sed -n '13,23p'   "$B2/pq1_parity.c"
  sed -n '119,147p' "$B2/pq1_parity.c"
  cat <<'EOF'
/* ---- exported wrappers (this repository's code) ---- */
float pbref_h2f(uint16_t h) { return pq1_h2f(h); }
void pbref_q1_repack(const uint8_t* q1, int rows, int K, uint32_t* wb, uint16_t* sc) { pq1_split_repack(q1, rows, K, wb, sc); }
void pbref_q1_gemv(int rows, int K, const uint32_t* wb, const uint16_t* sc, const uint8_t* xq, float* y) { pq1_gemv_cpu(rows, K, wb, sc, xq, y); }
uint16_t pbref_ff16(float f) { return ff16(f); }
float pbref_f16f(uint16_t h) { return f16f(h); }
void pbref_q80_quant(const float* x, int n, int8_t* q, float* d) { Q8 o = { q, d }; q8(x, n, &o); }
void pbref_mk_q8k(uint8_t* xq, int K, unsigned seed) { mk_q8k(xq, K, seed); }
void pbref_rms_q8k(float* x, const float* r, const float* w, int n, uint8_t* xq) { rms_ref(x, r, w, n, xq); }
/* the parity gate's weight generator (pq1_parity.c:750-758, restated) */
void pbref_parity_q1_weights(uint8_t* q1, int rows, int K) {
  const int nb = K / 128; const size_t q1b = (size_t)rows * nb * 18;
  srand(31337);
  for (size_t i = 0; i < q1b; i++) q1[i] = (uint8_t)(rand() & 0xFF);
  for (int r = 0; r < rows; r++)
    for (int b = 0; b < nb; b++) {
      uint16_t h = (uint16_t)(0x2800 + (rand() % 0x1000));
      memcpy(q1 + ((size_t)r * nb + b) * 18, &h, 2);
    }
}
EOF
} | "$CC" $CFL -x c -c -o "$out/pins_bonsai.o" -

# --- B: the x86/C CPU Q8 GEMV, whole file, main renamed ----------------------
{
  printf '#define main pbref_q8_gemv_cpu_main\n#include "%s"\n#undef main\n' "$REF/.auto/lfm3/q8_gemv_cpu.c"
  cat <<'EOF'
void pbref_gemv_q8(const signed char* q, const float* s, const float* x, float* y, int N, int K) { gemv_q8(q, s, x, y, N, K); }
void pbref_quant_row(const float* w, int K, signed char* q, float* s) { quant_row(w, K, q, s); }
EOF
} | "$CC" $CFL -x c -c -o "$out/pins_q8cpu.o" -

# --- C: cpuchk_run's scalar transcription of the tiled leaf order (C++) ------
{
  printf '#include <cstdint>\n#include <cstring>\n#include <cmath>\n#include <vector>\n'
  sed -n '4598,4603p' "$REF/pulsar_arm/asm/lfm3_nanode.cu"
  cat <<'EOF'
struct PbChk { long outs = 0, bad = 0; };
/* codes/scales row-major [N][K], [N][K/32] fp32; x bf16 [Tn][K]; y bf16 [Tn][N]
 * (the values under test). Tiles the last R rows the way lfm3_nanode.cu:4510-4521
 * does, then runs the reference's own loop; returns the bitwise-differ count. */
extern "C" long pbref_cpuchk(const int8_t* codes, const float* scales, const uint16_t* xb,
                             const uint16_t* yb, int N, int K, int Tn, int R) {
  const int nb = K / 32, r0 = N - R;
  const size_t tq = (size_t)nb * 64 * 16;
  std::vector<int8_t> hq((size_t)(R / 32) * tq);
  std::vector<float> hs((size_t)(R / 32) * nb * 32);
  for (int rr = 0; rr < R; rr++)
    for (int b = 0; b < nb; b++) {
      std::memcpy(&hq[(size_t)(rr >> 5) * tq + ((size_t)b * 64 + (rr & 31)) * 16], codes + (size_t)(r0 + rr) * K + b * 32, 16);
      std::memcpy(&hq[(size_t)(rr >> 5) * tq + ((size_t)b * 64 + 32 + (rr & 31)) * 16], codes + (size_t)(r0 + rr) * K + b * 32 + 16, 16);
      hs[(size_t)(rr >> 5) * nb * 32 + (size_t)b * 32 + (rr & 31)] = scales[(size_t)(r0 + rr) * nb + b];
    }
  std::vector<float> xf((size_t)Tn * K);
  for (size_t i = 0; i < xf.size(); i++) xf[i] = cpu_bf2f(xb[i]);
  std::vector<uint16_t> hy(yb, yb + (size_t)Tn * N);
  PbChk c;
EOF
  sed -n '4658,4684p' "$REF/pulsar_arm/asm/lfm3_nanode.cu"
  printf '  return c.bad;\n}\n'
} | "$CXX" -O2 -fPIC -ffp-contract=off -w -x c++ -c -o "$out/pins_cpuchk.o" -

# --- D: fwd8.c's rms and YaRN rope, built with gcc's default contraction as
#        the reference's own build is (8B constants, fwd8.c:51-57) -------------
{
  printf '#include <stdint.h>\n#include <math.h>\n#define YARN_FACTOR 4.0f\n#define YARN_ORIG 16384\n#define FREQ_BASE 1000000.0f\n'
  sed -n '312,317p' "$B2/fwd8.c"
  sed -n '320,369p' "$B2/fwd8.c"
  cat <<'EOF'
void pbref_bs_rms(const float* x, const float* w, int n, float* y) { rms(x, w, n, y); }
void pbref_bs_rope_table(int pos, float* c, float* s) {
  rope_table(pos);
  for (int j = 0; j < 64; j++) { c[j] = RC_C[j]; s[j] = RC_S[j]; }
}
void pbref_bs_rope(float* x, int heads, int pos) { rope_yarn_apply(x, heads, pos); }
EOF
} | "$CC" -O2 -fPIC -ffp-contract=fast -mfma -w -x c -c -o "$out/pins_fwd8.o" -

# --- E: pq1_host.c's f16 flash-attention decode and scalar silu tail, built
#        -ffp-contract=off as the reference builds that file; expf goes through
#        a hook (default libm) that the tests may point at the oracle's -----------
{
  printf '#include <stdint.h>\n#include <string.h>\n#include <math.h>\n#include <stddef.h>\n'
  printf 'float (*pbref_expf_hook)(float) = 0;\n'
  printf 'static float pbref_expf(float x) { return pbref_expf_hook ? pbref_expf_hook(x) : expf(x); }\n'
  printf '#define expf pbref_expf\n#define __fp16 _Float16\n'
  sed -n '373,434p' "$B2/pq1_host.c"
  printf 'void pbref_silu_mul(float* lu, const float* lg, int n) {\n  int i = 0;\n'
  sed -n '226p' "$B2/pq1_host.c"
  printf '}\n'
  printf 'void pbref_fa16_head(const float* q, const uint16_t* K, const uint16_t* V, int T, float scale, float* out) {\n'
  printf '  pq1_fa16_head(q, K, V, T, scale, out);\n}\n'
} | "$CC" $CFL -x c -c -o "$out/pins_fa16.o" -

"$CXX" -shared -fopenmp -o "$out/libpb_refpins.so" "$out/pins_bonsai.o" "$out/pins_q8cpu.o" "$out/pins_cpuchk.o" \
    "$out/pins_fwd8.o" "$out/pins_fa16.o" -lm
rm -f "$out"/pins_*.o
echo "build_ref: built $out/libpb_refpins.so"

# --- F: the reference's own LFM3 layer kernels (CUDA, sm_100a) --------------
#   lfm3_nanode.cu:74-83, 93     the compile-time shapes (H 2048, NH 16, NKV 4, HD 128, MAXTOK)
#   lfm3_nanode.cu:114-121       bf16 storage and its round-to-nearest-even pair
#   lfm3_nanode.cu:382-445       rmsnorm_body / k_rmsnorm
#   lfm3_nanode.cu:460-498       k_headnorm, k_rope
#   lfm3_nanode.cu:503-602       k_attn_head
#   lfm3_nanode.cu:811-829       k_mul_bf, k_add_bf, k_silu_mul_bf
#   lfm3_nanode.cu:852-859       k_sigmoid_gate
#   lfm3_nanode.cu:892-911       k_shift_in, k_conv7
#   lfm3_nanode.cu:942-964       k_argmax
#   lfm3_nanode.cu:164-167       k_bf2f
#   lfm3_nanode.cu:175-176       lfm_stage
#   lfm3_nanode.cu:222-343       q8_partial (the Q8 GEMV leaf) and k_combine_bf
#   lfm3_nanode.cu:3517-3534     k_gemv_bf16 (the certified arm's bf16 head)
# followed by host wrappers written here (host buffers in and out) and probes
# that return CUDA's own expf / rsqrtf / cosf / sinf for given arguments. The
# library runs on the GPU box only (tests/golden/make_golden_lfm3.py).
NVCC="${NVCC:-/usr/local/cuda/bin/nvcc}"
if [ -x "$NVCC" ]; then
  A="$REF/pulsar_arm/asm/lfm3_nanode.cu"
  {
    printf '#include <cstdint>\n#include <cstdio>\n#include <cmath>\n#include <cuda_runtime.h>\n#include <cuda_fp16.h>\n'
    sed -n '74,83p' "$A"
    sed -n '93p' "$A"
    sed -n '114,121p' "$A"
    sed -n '382,445p' "$A"
    sed -n '460,498p' "$A"
    sed -n '503,602p' "$A"
    sed -n '811,829p' "$A"
    sed -n '852,859p' "$A"
    sed -n '892,911p' "$A"
    sed -n '942,964p' "$A"
    sed -n '164,167p' "$A"
    sed -n '175,176p' "$A"
    sed -n '222,343p' "$A"
    sed -n '3517,3534p' "$A"
    cat <<'WRAP'
/* ---- host wrappers and probes (this repository's code) ---- */
namespace {
template <class T> T* up(const T* h, size_t n) { T* d = nullptr; cudaMalloc(&d, n * sizeof(T)); if (h) cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice); return d; }
template <class T> int down(T* h, const T* d, size_t n) { cudaMemcpy(h, d, n * sizeof(T), cudaMemcpyDeviceToHost); return cudaDeviceSynchronize() == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -1; }
__global__ void p_expf(const float* x, float* y, int n) { int i = blockIdx.x * blockDim.x + threadIdx.x; if (i < n) y[i] = expf(x[i]); }
__global__ void p_rsqrtf(const float* x, float* y, int n) { int i = blockIdx.x * blockDim.x + threadIdx.x; if (i < n) y[i] = rsqrtf(x[i]); }
__global__ void p_cossin(const float* x, float* c, float* s, int n) { int i = blockIdx.x * blockDim.x + threadIdx.x; if (i < n) { c[i] = cosf(x[i]); s[i] = sinf(x[i]); } }
}
extern "C" {
int pbref_shapes(int* o) { o[0] = H; o[1] = NH; o[2] = NKV; o[3] = HD; o[4] = MAXTOK; return 0; }
int pbref_gpu_rmsnorm(const uint16_t* x, const float* w, uint16_t* y, float eps) {
  bf16* dx = up((const bf16*)x, H); float* dw = up(w, H); bf16* dy = up((const bf16*)nullptr, H);
  k_rmsnorm<<<1, 256>>>(dx, dw, dy, eps, H);
  int rc = down((bf16*)y, dy, H); cudaFree(dx); cudaFree(dw); cudaFree(dy); return rc;
}
int pbref_gpu_headnorm(uint16_t* x, const float* w, int nheads, float eps) {
  bf16* dx = up((const bf16*)x, (size_t)nheads * HD); float* dw = up(w, HD);
  k_headnorm<<<nheads, 32>>>(dx, dw, eps, HD);
  int rc = down((bf16*)x, dx, (size_t)nheads * HD); cudaFree(dx); cudaFree(dw); return rc;
}
int pbref_gpu_rope(uint16_t* x, const float* invf, int nheads, int pos, int rot) {
  bf16* dx = up((const bf16*)x, (size_t)nheads * HD); float* di = up(invf, HD / 2);
  k_rope<<<nheads, 64>>>(dx, di, pos, HD, rot);
  int rc = down((bf16*)x, dx, (size_t)nheads * HD); cudaFree(dx); cudaFree(di); return rc;
}
/* q [NH][HD]; kc, vc [npos][NKV][HD]; out [NH][HD] */
int pbref_gpu_attn(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* out, int npos, int win,
                   float scaling) {
  bf16* dq = up((const bf16*)q, (size_t)NH * HD);
  bf16* dk = up((const bf16*)kc, (size_t)npos * NKV * HD);
  bf16* dv = up((const bf16*)vc, (size_t)npos * NKV * HD);
  bf16* dout = up((const bf16*)nullptr, (size_t)NH * HD);
  k_attn_head<<<NH, 256>>>(dq, dk, dv, dout, npos, win, scaling, HD, NKV);
  int rc = down((bf16*)out, dout, (size_t)NH * HD); cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout); return rc;
}
int pbref_gpu_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* y, int n) {
  bf16* da = up((const bf16*)a, n); bf16* db = up((const bf16*)b, n); bf16* dy = up((const bf16*)nullptr, n);
  k_silu_mul_bf<<<(n + 255) / 256, 256>>>(da, db, dy, n);
  int rc = down((bf16*)y, dy, n); cudaFree(da); cudaFree(db); cudaFree(dy); return rc;
}
int pbref_gpu_mul_bf(const uint16_t* a, const uint16_t* b, uint16_t* y, int n) {
  bf16* da = up((const bf16*)a, n); bf16* db = up((const bf16*)b, n); bf16* dy = up((const bf16*)nullptr, n);
  k_mul_bf<<<(n + 255) / 256, 256>>>(da, db, dy, n);
  int rc = down((bf16*)y, dy, n); cudaFree(da); cudaFree(db); cudaFree(dy); return rc;
}
/* g [nh]; attn [nh][HD] gated in place */
int pbref_gpu_sigmoid_gate(const uint16_t* g, uint16_t* attn, int nh) {
  bf16* dg = up((const bf16*)g, nh); bf16* da = up((const bf16*)attn, (size_t)nh * HD);
  k_sigmoid_gate<<<1, nh>>>(dg, da, HD);
  int rc = down((bf16*)attn, da, (size_t)nh * HD); cudaFree(dg); cudaFree(da); return rc;
}
/* ring [7][H] (newest last) shifted in place with xin [H]; y [H] = the conv */
int pbref_gpu_conv(uint16_t* ring, const uint16_t* xin, const float* taps, uint16_t* y) {
  bf16* dr = up((const bf16*)ring, (size_t)7 * H); bf16* dx = up((const bf16*)xin, H);
  float* dt = up(taps, (size_t)H * 7); bf16* dy = up((const bf16*)nullptr, H);
  k_shift_in<<<H / 256, 256>>>(dr, dx, H);
  k_conv7<<<H / 256, 256>>>(dr, dt, dy, H);
  int rc = down((bf16*)y, dy, H); if (!rc) rc = down((bf16*)ring, dr, (size_t)7 * H);
  cudaFree(dr); cudaFree(dx); cudaFree(dt); cudaFree(dy); return rc;
}
int pbref_gpu_argmax(const float* lg, int n, int* out) {
  float* dl = up(lg, n); int* di = up((const int*)nullptr, 1);
  k_argmax<<<1, 256>>>(dl, di, n);
  int rc = down(out, di, 1); cudaFree(dl); cudaFree(di); return rc;
}
/* y = bf16(gemv): q8_partial<bf16, FMA=true> with pick()'s KCHUNK (2048 when
   it divides K, else K) and R (256 from N 1024, else 64), then k_combine_bf */
int pbref_gpu_q8_gemv(const int8_t* q, const float* s, const uint16_t* x, uint16_t* y, int N, int K) {
  const int KC = (K >= 2048 && K % 2048 == 0) ? 2048 : K, nch = K / KC, R = N >= 1024 ? 256 : 64;
  int8_t* dq = up(q, (size_t)N * K); float* ds = up(s, (size_t)N * (K / 32));
  bf16* dx = up((const bf16*)x, K); float* dp = up((const float*)nullptr, (size_t)N * nch);
  bf16* dy = up((const bf16*)nullptr, N);
  const size_t shm = (size_t)(KC / 32) * 33 * sizeof(float);
  cudaFuncSetAttribute(q8_partial<bf16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm);
  q8_partial<bf16, true><<<((N + R - 1) / R) * nch, 256, shm>>>(dq, ds, dx, dp, N, K, KC, R, KC / 32);
  k_combine_bf<<<(N + 255) / 256, 256>>>(dp, dy, N, nch);
  int rc = down((bf16*)y, dy, N);
  cudaFree(dq); cudaFree(ds); cudaFree(dx); cudaFree(dp); cudaFree(dy); return rc;
}
/* mean microseconds of pbref_gpu_q8_gemv's two launches over `reps` calls,
   cycling over `ncopy` device copies of the tensor (together larger than L2),
   CUDA events after one warm pass */
float pbref_gpu_q8_gemv_time(const int8_t* q, const float* s, int N, int K, int ncopy, int reps) {
  const int KC = (K >= 2048 && K % 2048 == 0) ? 2048 : K, nch = K / KC, R = N >= 1024 ? 256 : 64;
  const size_t nq = (size_t)N * K, nsc = (size_t)N * (K / 32);
  int8_t* dq = up((const int8_t*)nullptr, nq * ncopy); float* ds = up((const float*)nullptr, nsc * ncopy);
  for (int c = 0; c < ncopy; c++) { cudaMemcpy(dq + nq * c, q, nq, cudaMemcpyHostToDevice); cudaMemcpy(ds + nsc * c, s, nsc * 4, cudaMemcpyHostToDevice); }
  bf16* dx = up((const bf16*)nullptr, K); float* dp = up((const float*)nullptr, (size_t)N * nch);
  bf16* dy = up((const bf16*)nullptr, N);
  cudaMemset(dx, 0, (size_t)K * 2);
  const size_t shm = (size_t)(KC / 32) * 33 * sizeof(float);
  cudaFuncSetAttribute(q8_partial<bf16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)shm);
  auto run = [&](int c) {
    q8_partial<bf16, true><<<((N + R - 1) / R) * nch, 256, shm>>>(dq + nq * c, ds + nsc * c, dx, dp, N, K, KC, R, KC / 32);
    k_combine_bf<<<(N + 255) / 256, 256>>>(dp, dy, N, nch);
  };
  for (int c = 0; c < ncopy; c++) run(c);
  cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  for (int r = 0; r < reps; r++) for (int c = 0; c < ncopy; c++) run(c);
  cudaEventRecord(e1); cudaEventSynchronize(e1);
  float ms = 0.f; cudaEventElapsedTime(&ms, e0, e1);
  const int ok = cudaGetLastError() == cudaSuccess;
  cudaFree(dq); cudaFree(ds); cudaFree(dx); cudaFree(dp); cudaFree(dy); cudaEventDestroy(e0); cudaEventDestroy(e1);
  return ok ? ms * 1e3f / (reps * ncopy) : -1.0f;
}
/* logits = lm_head_bf16: k_bf2f of x, k_gemv_bf16 with R = 32 rows per block */
int pbref_gpu_gemv_bf16(const uint16_t* w, const uint16_t* x, float* y, int N, int K) {
  bf16* dw = up((const bf16*)w, (size_t)N * K); bf16* dx = up((const bf16*)x, K);
  float* dxf = up((const float*)nullptr, K); float* dy = up((const float*)nullptr, N);
  k_bf2f<<<(K + 255) / 256, 256>>>(dx, dxf, K);
  k_gemv_bf16<<<(N + 31) / 32, 256, (size_t)K * sizeof(float)>>>(dw, dxf, dy, N, K, 32);
  int rc = down(y, dy, N);
  cudaFree(dw); cudaFree(dx); cudaFree(dxf); cudaFree(dy); return rc;
}
int pbref_gpu_expf(const float* x, float* y, int n) {
  float* dx = up(x, n); float* dy = up((const float*)nullptr, n);
  p_expf<<<(n + 255) / 256, 256>>>(dx, dy, n);
  int rc = down(y, dy, n); cudaFree(dx); cudaFree(dy); return rc;
}
int pbref_gpu_rsqrtf(const float* x, float* y, int n) {
  float* dx = up(x, n); float* dy = up((const float*)nullptr, n);
  p_rsqrtf<<<(n + 255) / 256, 256>>>(dx, dy, n);
  int rc = down(y, dy, n); cudaFree(dx); cudaFree(dy); return rc;
}
int pbref_gpu_cossin(const float* x, float* c, float* s, int n) {
  float* dx = up(x, n); float* dc = up((const float*)nullptr, n); float* ds = up((const float*)nullptr, n);
  p_cossin<<<(n + 255) / 256, 256>>>(dx, dc, ds, n);
  int rc = down(c, dc, n); if (!rc) rc = down(s, ds, n); cudaFree(dx); cudaFree(dc); cudaFree(ds); return rc;
}
}
WRAP
  } > "$out/refgpu.cu"
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared -w \
      -o "$out/libpb_refgpu.so" "$out/refgpu.cu"
  rm -f "$out/refgpu.cu"
  echo "build_ref: built $out/libpb_refgpu.so"
fi

# --- F2: the reference's low-bit GEMV kernels (pulsar_arm/asm/lfm3_qlow.cuh,
#         included where it lies: k_qlow + k_qlow_combine), with a wrapper
#         written here that launches them as qlow_gemv does
#         (lfm3_nanode.cu:1898-1915: KS 2, 4 from K = 4096; PD 2 at 4 blocks per
#         SM, the default) on host buffers. GPU box only
#         (tests/golden/make_golden_qlow.py).
if [ -x "$NVCC" ]; then
  {
    printf '#include <cstdint>\n#include <cuda_runtime.h>\n#include "%s"\n' "$REF/pulsar_arm/asm/lfm3_qlow.cuh"
    cat <<'WRAP'
/* ---- host wrapper (this repository's code) ---- */
extern "C" int pbref_gpu_qlow(const void* q, const void* s, int bits, const uint16_t* x, uint16_t* y, int N, int K) {
  const size_t nc = (size_t)N * K / 32 * (bits == 5 ? 20 : 16), ns = (size_t)N * K / 32 * 4;
  const int KS = K >= 4096 ? 4 : 2;
  const size_t sm = (size_t)(K / KS + K / 32 / KS) * 4;
  void *dq, *ds, *dx, *dy, *dp;
  cudaMalloc(&dq, nc); cudaMalloc(&ds, ns); cudaMalloc(&dx, (size_t)K * 2); cudaMalloc(&dy, (size_t)N * 2);
  cudaMalloc(&dp, (size_t)KS * N * 4);
  cudaMemcpy(dq, q, nc, cudaMemcpyHostToDevice); cudaMemcpy(ds, s, ns, cudaMemcpyHostToDevice);
  cudaMemcpy(dx, x, (size_t)K * 2, cudaMemcpyHostToDevice);
  const dim3 gr((unsigned)((N + 255) / 256), (unsigned)KS);
  const uint4* cq = (const uint4*)dq; const __half2* cs = (const __half2*)ds;
  if (bits == 4) k_qlow<4, 256, 2, 4><<<gr, 256, sm>>>(cq, cs, (const unsigned short*)dx, (float*)dp, (unsigned short*)dy, N, K);
  else           k_qlow<5, 256, 2, 4><<<gr, 256, sm>>>(cq, cs, (const unsigned short*)dx, (float*)dp, (unsigned short*)dy, N, K);
  k_qlow_combine<<<(N + 255) / 256, 256>>>((const float*)dp, (unsigned short*)dy, N, KS);
  cudaMemcpy(y, dy, (size_t)N * 2, cudaMemcpyDeviceToHost);
  const int rc = cudaDeviceSynchronize() == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -1;
  cudaFree(dq); cudaFree(ds); cudaFree(dx); cudaFree(dy); cudaFree(dp);
  return rc;
}
/* mean microseconds of qlow_gemv's two launches over `reps` calls, cycling
   over `ncopy` device copies of the tensor (together larger than L2), timed
   with CUDA events after one warm pass */
extern "C" float pbref_gpu_qlow_time(const void* q, const void* s, int bits, int N, int K, int ncopy, int reps) {
  const size_t nc = (size_t)N * K / 32 * (bits == 5 ? 20 : 16), ns = (size_t)N * K / 32 * 4;
  const int KS = K >= 4096 ? 4 : 2;
  const size_t sm = (size_t)(K / KS + K / 32 / KS) * 4;
  char *dq, *ds; void *dx, *dy, *dp;
  cudaMalloc(&dq, nc * ncopy); cudaMalloc(&ds, ns * ncopy); cudaMalloc(&dx, (size_t)K * 2); cudaMalloc(&dy, (size_t)N * 2);
  cudaMalloc(&dp, (size_t)KS * N * 4); cudaMemset(dx, 0, (size_t)K * 2);
  for (int c = 0; c < ncopy; c++) { cudaMemcpy(dq + nc * c, q, nc, cudaMemcpyHostToDevice); cudaMemcpy(ds + ns * c, s, ns, cudaMemcpyHostToDevice); }
  const dim3 gr((unsigned)((N + 255) / 256), (unsigned)KS);
  auto run = [&](int c) {
    const uint4* cq = (const uint4*)(dq + nc * c); const __half2* cs = (const __half2*)(ds + ns * c);
    if (bits == 4) k_qlow<4, 256, 2, 4><<<gr, 256, sm>>>(cq, cs, (const unsigned short*)dx, (float*)dp, (unsigned short*)dy, N, K);
    else           k_qlow<5, 256, 2, 4><<<gr, 256, sm>>>(cq, cs, (const unsigned short*)dx, (float*)dp, (unsigned short*)dy, N, K);
    k_qlow_combine<<<(N + 255) / 256, 256>>>((const float*)dp, (unsigned short*)dy, N, KS);
  };
  for (int c = 0; c < ncopy; c++) run(c);
  cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
  cudaEventRecord(e0);
  for (int r = 0; r < reps; r++) for (int c = 0; c < ncopy; c++) run(c);
  cudaEventRecord(e1); cudaEventSynchronize(e1);
  float ms = 0.f; cudaEventElapsedTime(&ms, e0, e1);
  const int ok = cudaGetLastError() == cudaSuccess;
  cudaFree(dq); cudaFree(ds); cudaFree(dx); cudaFree(dy); cudaFree(dp); cudaEventDestroy(e0); cudaEventDestroy(e1);
  return ok ? ms * 1e3f / (reps * ncopy) : -1.0f;
}
WRAP
  } > "$out/refqlow.cu"
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared -w \
      -o "$out/libpb_refqlow.so" "$out/refqlow.cu"
  rm -f "$out/refqlow.cu"
  echo "build_ref: built $out/libpb_refqlow.so"
fi

# --- F3: the reference's TurboQuant K/V kernels (pulsar_arm/bonsai2/
#         pq1_swar_sm53.cu, cut by line range and compiled where they lie):
#   :2164        PQ1_APAR_NPOS (the parameter block's position slot)
#   :2187-2191   pq1_h2f
#   :3264-3376   codebook, thresholds, sign pattern, pq1_fwht128, pq1_tq_row,
#                pq1_tq_store
#   :3447-3550   pq1_tq_qk2, pq1_tq_sm
#   :3619-3689   pq1_tq_pv2
#   :3698-3715   pq1_tq_out
#   :3716-3906   pq1_tq_qks, pq1_tq_tail (the short pair)
# with host wrappers written here (host buffers in and out). GPU box only
# (tests/golden/make_golden_tq.py).
if [ -x "$NVCC" ]; then
  S="$REF/pulsar_arm/bonsai2/pq1_swar_sm53.cu"
  {
    printf '#include <cstdint>\n#include <cmath>\n#include <cuda_runtime.h>\n#include <cuda_fp16.h>\n'
    sed -n '2164p' "$S"
    sed -n '2187,2191p' "$S"
    sed -n '3264,3376p' "$S"
    sed -n '3447,3550p' "$S"
    sed -n '3619,3689p' "$S"
    sed -n '3698,3715p' "$S"
    sed -n '3716,3906p' "$S"
    cat <<'WRAP'
/* ---- host wrappers (this repository's code) ---- */
namespace {
template <class T> T* tup(const T* h, size_t n) { T* d = nullptr; cudaMalloc(&d, n * sizeof(T) + 16); if (h) cudaMemcpy(d, h, n * sizeof(T), cudaMemcpyHostToDevice); else cudaMemset(d, 0, n * sizeof(T) + 16); return d; }
template <class T> int tdown(T* h, const T* d, size_t n) { cudaMemcpy(h, d, n * sizeof(T), cudaMemcpyDeviceToHost); return cudaDeviceSynchronize() == cudaSuccess && cudaGetLastError() == cudaSuccess ? 0 : -1; }
int cwof(int b) { return b == 3 ? 12 : 16; }
}
extern "C" {
/* encode 2 nkv f16 rows (nkv K rows, then nkv V rows) with pq1_tq_store at
   bits bk (K) / bv (V): K codes [nkv][CW(bk)], scales [nkv]; V alike */
int pbref_gpu_tq_store(const uint16_t* rows, int nkv, int bk, int bv, uint32_t* kcw, float* ksc, uint32_t* vcw, float* vsc) {
  unsigned short* ds = tup((const unsigned short*)rows, (size_t)2 * nkv * 128);
  uint32_t* dk = tup((const uint32_t*)nullptr, (size_t)nkv * cwof(bk)); float* dks = tup((const float*)nullptr, nkv);
  uint32_t* dv = tup((const uint32_t*)nullptr, (size_t)nkv * cwof(bv)); float* dvs = tup((const float*)nullptr, nkv);
  if (bk == 3 && bv == 3) pq1_tq_store<3, 3><<<1, 64 * nkv>>>(ds, nullptr, 0, dk, dks, dv, dvs, nkv, 1);
  else if (bk == 4 && bv == 4) pq1_tq_store<4, 4><<<1, 64 * nkv>>>(ds, nullptr, 0, dk, dks, dv, dvs, nkv, 1);
  else pq1_tq_store<4, 3><<<1, 64 * nkv>>>(ds, nullptr, 0, dk, dks, dv, dvs, nkv, 1);
  int rc = tdown(kcw, dk, (size_t)nkv * cwof(bk)); if (!rc) rc = tdown(ksc, dks, nkv);
  if (!rc) rc = tdown(vcw, dv, (size_t)nkv * cwof(bv)); if (!rc) rc = tdown(vsc, dvs, nkv);
  cudaFree(ds); cudaFree(dk); cudaFree(dks); cudaFree(dv); cudaFree(dvs); return rc;
}
/* the long chain (pq1_tq_qk2, pq1_tq_sm, pq1_tq_pv2, pq1_tq_out) over
   positions 0..T-1 of caches with position stride ctx: q [4 nkv][128] fp32,
   K codes [nkv][ctx][CW], scales [nkv][ctx], V alike; atto [4 nkv][128] */
int pbref_gpu_tq_attn(const float* q, int bk, int bv, const uint32_t* kcw, const float* ksc, const uint32_t* vcw,
                      const float* vsc, int nkv, int ctx, int T, float* atto) {
  const int nh = 4 * nkv, npos = T - 1;
  uint8_t par[1024] = {0}; *reinterpret_cast<int*>(par + PQ1_APAR_NPOS) = npos;
  uint8_t* dp = tup(par, sizeof par); float* dq = tup(q, (size_t)nh * 128);
  uint32_t* dk = tup(kcw, (size_t)nkv * ctx * cwof(bk)); float* dks = tup(ksc, (size_t)nkv * ctx);
  uint32_t* dv = tup(vcw, (size_t)nkv * ctx * cwof(bv)); float* dvs = tup(vsc, (size_t)nkv * ctx);
  float* dsc = tup((const float*)nullptr, (size_t)nh * ctx); float* dinv = tup((const float*)nullptr, nh);
  const int nch = (ctx + PQ1_TQ_CH - 1) / PQ1_TQ_CH;
  float* dpart = tup((const float*)nullptr, (size_t)nch * nh * 128); float* dat = tup((const float*)nullptr, (size_t)nh * 128);
  const dim3 gq(nkv, (ctx + 511) / 512 < PQ1_TQ_QB ? (ctx + 511) / 512 : PQ1_TQ_QB), gp(nkv, nch);
  if (bk == 3) pq1_tq_qk2<3><<<gq, 256>>>(dq, dk, dks, dp, dsc, ctx); else pq1_tq_qk2<4><<<gq, 256>>>(dq, dk, dks, dp, dsc, ctx);
  pq1_tq_sm<<<nh, 256>>>(dsc, dp, dinv, ctx);
  if (bv == 3) pq1_tq_pv2<3><<<gp, 128>>>(dsc, dv, dvs, dp, dpart, nh, ctx); else pq1_tq_pv2<4><<<gp, 128>>>(dsc, dv, dvs, dp, dpart, nh, ctx);
  pq1_tq_out<<<nh, 32>>>(dpart, dinv, dp, dat, nh);
  int rc = tdown(atto, dat, (size_t)nh * 128);
  cudaFree(dp); cudaFree(dq); cudaFree(dk); cudaFree(dks); cudaFree(dv); cudaFree(dvs); cudaFree(dsc); cudaFree(dinv);
  cudaFree(dpart); cudaFree(dat); return rc;
}
/* the short pair (pq1_tq_qks encodes the staged rows of position T-1 into the
   caches, pq1_tq_tail) for T <= 256: stage [2 nkv][128] f16; the caches are
   read and updated; atto as above */
int pbref_gpu_tq_short(const float* q, const uint16_t* stage, int bk, int bv, uint32_t* kcw, float* ksc, uint32_t* vcw,
                       float* vsc, int nkv, int ctx, int T, float* atto) {
  const int nh = 4 * nkv, npos = T - 1;
  uint8_t par[1024] = {0}; *reinterpret_cast<int*>(par + PQ1_APAR_NPOS) = npos;
  uint8_t* dp = tup(par, sizeof par); float* dq = tup(q, (size_t)nh * 128);
  unsigned short* dst = tup((const unsigned short*)stage, (size_t)2 * nkv * 128);
  uint32_t* dk = tup(kcw, (size_t)nkv * ctx * cwof(bk)); float* dks = tup(ksc, (size_t)nkv * ctx);
  uint32_t* dv = tup(vcw, (size_t)nkv * ctx * cwof(bv)); float* dvs = tup(vsc, (size_t)nkv * ctx);
  float* dsc = tup((const float*)nullptr, (size_t)nh * ctx); float* dat = tup((const float*)nullptr, (size_t)nh * 128);
  const dim3 g(nkv, ((ctx < PQ1_TQ_CH ? ctx : PQ1_TQ_CH) + PQ1_TQ_SB - 1) / PQ1_TQ_SB);
  if (bk == 3 && bv == 3) { pq1_tq_qks<3, 3><<<g, PQ1_TQ_SB>>>(dq, dst, dp, dk, dks, dv, dvs, dsc, nkv, ctx); pq1_tq_tail<3><<<nkv, 256>>>(dsc, dv, dvs, dp, dat, ctx); }
  else if (bk == 4 && bv == 4) { pq1_tq_qks<4, 4><<<g, PQ1_TQ_SB>>>(dq, dst, dp, dk, dks, dv, dvs, dsc, nkv, ctx); pq1_tq_tail<4><<<nkv, 256>>>(dsc, dv, dvs, dp, dat, ctx); }
  else { pq1_tq_qks<4, 3><<<g, PQ1_TQ_SB>>>(dq, dst, dp, dk, dks, dv, dvs, dsc, nkv, ctx); pq1_tq_tail<3><<<nkv, 256>>>(dsc, dv, dvs, dp, dat, ctx); }
  int rc = tdown(atto, dat, (size_t)nh * 128);
  if (!rc) rc = tdown(kcw, dk, (size_t)nkv * ctx * cwof(bk)); if (!rc) rc = tdown(ksc, dks, (size_t)nkv * ctx);
  if (!rc) rc = tdown(vcw, dv, (size_t)nkv * ctx * cwof(bv)); if (!rc) rc = tdown(vsc, dvs, (size_t)nkv * ctx);
  cudaFree(dp); cudaFree(dq); cudaFree(dst); cudaFree(dk); cudaFree(dks); cudaFree(dv); cudaFree(dvs); cudaFree(dsc); cudaFree(dat);
  return rc;
}
}
WRAP
  } > "$out/reftq.cu"
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared -w \
      -o "$out/libpb_reftq.so" "$out/reftq.cu"
  rm -f "$out/reftq.cu"
  echo "build_ref: built $out/libpb_reftq.so"
fi

# --- G: the reference's x86/C CPU Q8 GEMV, unmodified, for timing: its own
#        flags (.auto/lfm3/q8_gemv_cpu.c:16, -fopenmp -ffp-contract=off) at -O3,
#        once for the baseline x86-64 ISA and once for x86-64-v3 (AVX2); the
#        second arm stands in for -march=native because this build runs off the
#        GPU box, whose host CPU may differ. Timed by bench.py (cpu_reference).
Q8C="$REF/.auto/lfm3/q8_gemv_cpu.c"
for arm in O3 v3; do
  extra=""; [ "$arm" = v3 ] && extra="-march=x86-64-v3"
  {
    printf '#define main pbref_q8_gemv_cpu_main\n#include "%s"\n#undef main\n' "$Q8C"
    cat <<'WRAP'
void pbref_gemv_q8(const signed char* q, const float* s, const float* x, float* y, int N, int K) { gemv_q8(q, s, x, y, N, K); }
void pbref_quant_row(const float* w, int K, signed char* q, float* s) { quant_row(w, K, q, s); }
void pbref_set_threads(int n) { omp_set_num_threads(n); }
WRAP
  } | "$CC" -O3 -fPIC -fopenmp -ffp-contract=off -w $extra -shared -x c -o "$out/libpb_q8cpu_$arm.so" - -lm
  echo "build_ref: built $out/libpb_q8cpu_$arm.so"
done

# --- H: fwd8.c's GGUF table reader (pulsar_arm/bonsai2/fwd8.c:205-245:
#        the table statics and gguf_table), unmodified, with a lookup wrapper
#        written here; tests/test_export.py compares pulsar_b200.gguf's
#        tensor offsets with it.
F8="$REF/pulsar_arm/bonsai2/fwd8.c"
{
  printf '#include <stdio.h>\n#include <stdint.h>\n#include <stdlib.h>\n#include <string.h>\n#include <fcntl.h>\n#include <sys/mman.h>\n#include <sys/stat.h>\n#include <unistd.h>\n'
  sed -n '205,245p' "$F8"
  cat <<'WRAP'
/* ---- lookup wrapper (this repository's code) ---- */
int pbref_gguf_offset(const char* path, const char* name, unsigned long long* off) {
  static char opened[4096];
  if (strcmp(opened, path)) { gguf_table(path); strncpy(opened, path, sizeof opened - 1); }
  for (int i = 0; i < NT; i++)
    if (!strcmp(TN[i], name)) { *off = (unsigned long long)TO[i]; return 0; }
  return -1;
}
WRAP
} | "$CC" -O2 -fPIC -shared -w -x c -o "$out/libpb_gguf.so" -
echo "build_ref: built $out/libpb_gguf.so"

# --- I: fwd8.c's sampler (pulsar_arm/bonsai2/fwd8.c:465-521: argmax, the
#        generator state RS, frand01 and sample_topkpp), unmodified, built with
#        gcc's default contraction as D is, with a wrapper written here that
#        loads and returns the generator state; tests/test_sample.py compares
#        the oracle's restatement with it.
{
  printf '#include <stdint.h>\n#include <math.h>\n'
  sed -n '465,521p' "$F8"
  cat <<'WRAP'
/* ---- wrapper (this repository's code) ---- */
int pbref_sample_topkpp(const float* lg, int n, float temp, float topp, int topk, float minp, uint64_t* rs) {
  RS = *rs;
  const int id = sample_topkpp(lg, n, temp, topp, topk, minp);
  *rs = RS;
  return id;
}
WRAP
} | "$CC" -O2 -fPIC -shared -ffp-contract=fast -mfma -w -x c -o "$out/libpb_sample.so" - -lm
echo "build_ref: built $out/libpb_sample.so"
