/* q4k_oracle.c -- CPU restatement of the k-quant dequant + sequential fp32 MAC contract
 * (TEST INFRASTRUCTURE ONLY: the checker and the timed CPU baseline, never the product).
 *
 * Restates Wick-Lim/AIPU tools/q4k_ref.py:
 *   dequantize_block_q4_K  q4k_ref.py:39-61   w = (d*sc)*q - (dmin*m), each op rounded
 *   get_scale_min_k4       q4k_ref.py:27-37
 *   dequantize_block_q6_K  q4k_ref.py:105-124 w = (d*f32(int8 sc))*f32(q-32)
 *   dequantize_block_q8_0  q4k_ref.py:126-129 w = d*f32(int8 q)
 *   matmul_q4k_col         q4k_ref.py:86-92   acc = f32(acc + f32(a*w)) in K order, bf16 RNE
 * Built with -ffp-contract=off so no product/sum pair is fused (the reference rounds each op).
 * Rows are split across POSIX threads; each output is still one sequential chain, so the result is
 * bit-identical to the scalar reference for any thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float f16_to_f32(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF, u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else { /* subnormal: normalise */
      int sh = 0;
      while (!(m & 0x400)) { m <<= 1; ++sh; }
      m &= 0x3FF;
      u = s | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
    }
  } else if (e == 0x1F) {
    u = s | 0x7F800000u | (m << 13);
  } else {
    u = s | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t bf16_rne(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

static void scale_min(const uint8_t* q, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

static int64_t row_bytes(int wt, int64_t K) {
  switch (wt) {
    case 0: return K / 256 * 144;
    case 1: return K / 256 * 210;
    case 2: return K / 32 * 34;
    case 3: return K * 2;
    default: return K * 4;
  }
}

/* exact dequant of one row of K weights */
void oracle_dequant_row(int wt, const uint8_t* row, int64_t K, float* out) {
  if (wt == 0) {
    for (int64_t sb = 0; sb < K / 256; ++sb) {
      const uint8_t* b = row + sb * 144;
      float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8))), dmin = f16_to_f32((uint16_t)(b[2] | (b[3] << 8)));
      for (int g = 0; g < 4; ++g) {
        int sc, m;
        scale_min(b + 4, 2 * g, &sc, &m);
        float d1 = d * (float)sc, m1 = dmin * (float)m;
        scale_min(b + 4, 2 * g + 1, &sc, &m);
        float d2 = d * (float)sc, m2 = dmin * (float)m;
        const uint8_t* qs = b + 16 + 32 * g;
        float* y = out + sb * 256 + 64 * g;
        for (int l = 0; l < 32; ++l) {
          float t = d1 * (float)(qs[l] & 0xF);
          y[l] = t - m1;
        }
        for (int l = 0; l < 32; ++l) {
          float t = d2 * (float)(qs[l] >> 4);
          y[32 + l] = t - m2;
        }
      }
    }
  } else if (wt == 1) {
    for (int64_t sb = 0; sb < K / 256; ++sb) {
      const uint8_t* b = row + sb * 210;
      float d = f16_to_f32((uint16_t)(b[208] | (b[209] << 8)));
      const int8_t* sc = (const int8_t*)(b + 192);
      for (int hf = 0; hf < 2; ++hf) {
        const uint8_t* ql = b + 64 * hf;
        const uint8_t* qh = b + 128 + 32 * hf;
        float* y = out + sb * 256 + 128 * hf;
        for (int l = 0; l < 32; ++l) {
          int is = l / 16;
          int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
          int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
          int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
          int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
          float s1 = d * (float)sc[8 * hf + is + 0], s2 = d * (float)sc[8 * hf + is + 2];
          float s3 = d * (float)sc[8 * hf + is + 4], s4 = d * (float)sc[8 * hf + is + 6];
          y[l] = s1 * (float)q1;
          y[l + 32] = s2 * (float)q2;
          y[l + 64] = s3 * (float)q3;
          y[l + 96] = s4 * (float)q4;
        }
      }
    }
  } else if (wt == 2) {
    for (int64_t bi = 0; bi < K / 32; ++bi) {
      const uint8_t* b = row + bi * 34;
      float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
      for (int l = 0; l < 32; ++l) out[bi * 32 + l] = d * (float)(int8_t)b[2 + l];
    }
  } else if (wt == 3) {
    for (int64_t k = 0; k < K; ++k) out[k] = f16_to_f32((uint16_t)(row[2 * k] | (row[2 * k + 1] << 8)));
  } else {
    memcpy(out, row, (size_t)K * 4);
  }
}

typedef struct {
  int wt;
  const uint8_t* w;
  int64_t N, K;
  const float* x;
  int64_t M;
  uint16_t* y;
  int64_t r0, r1;
} job_t;

#define RB 8 /* rows interleaved per chain group (independent chains, still sequential in k) */

static void* run_rows(void* arg) {
  job_t* j = (job_t*)arg;
  const int64_t K = j->K, rb = row_bytes(j->wt, K);
  float* wd = (float*)calloc((size_t)K * RB, sizeof(float));
  for (int64_t n0 = j->r0; n0 < j->r1; n0 += RB) {
    int nr = (int)((j->r1 - n0) < RB ? (j->r1 - n0) : RB);
    for (int r = 0; r < nr; ++r) oracle_dequant_row(j->wt, j->w + (n0 + r) * rb, K, wd + (int64_t)r * K);
    for (int64_t m = 0; m < j->M; ++m) {
      const float* xm = j->x + m * K;
      float acc[RB] = {0};
      for (int64_t k = 0; k < K; ++k) {
        const float a = xm[k];
        for (int r = 0; r < RB; ++r) {
          float p = a * wd[(int64_t)r * K + k];
          acc[r] = acc[r] + p;
        }
      }
      for (int r = 0; r < nr; ++r) j->y[m * j->N + n0 + r] = bf16_rne(acc[r]);
    }
  }
  free(wd);
  return NULL;
}

/* y[M, N] (bf16 bits) = sequential-contract GEMM of fp32 x[M, K] with N rows of type wt */
int oracle_gemm(int wt, const uint8_t* w, int64_t N, int64_t K, const float* x, int64_t M, uint16_t* y,
                int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 512) nthreads = 512;
  pthread_t th[512];
  job_t jobs[512];
  int64_t per = (N + nthreads - 1) / nthreads;
  per = (per + RB - 1) / RB * RB;
  int nt = 0;
  for (int t = 0; t < nthreads; ++t) {
    int64_t r0 = t * per, r1 = r0 + per < N ? r0 + per : N;
    if (r0 >= N) break;
    jobs[nt] = (job_t){wt, w, N, K, x, M, y, r0, r1};
    if (pthread_create(&th[nt], NULL, run_rows, &jobs[nt]) != 0) return -1;
    ++nt;
  }
  for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
  return 0;
}
