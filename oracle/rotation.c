/*
 * ORACLE (test infrastructure only; never linked into the product library).
 *
 * CPU restatement of the reference's group-256 Hadamard rotation
 *   slimdit/hadamard.py:45-58   rotate(): np.matmul(W.reshape(N, K/256, 256), H.T)
 *   slimdit/hadamard.py:18-42   H = kron^4(H4) / sqrt(256), H4[a][b] = -1 iff a + b == 3
 * in the exact fp32 summation orders that numpy 2.3.5 + OpenBLAS 0.3.30 (x86-64, SkylakeX
 * kernels) execute for it: one sgemm [G,256]x[256,256] per row, G = K/256, with
 *   G >= 5      one sequential chain over k = 0..255                     (sgemm kernel)
 *   2 <= G <= 4 16 chains over k mod 16, then pairwise tree (0+1, 2+3..) (small-matrix kernel)
 *   G == 1      8 chains over k mod 8, then c_i + c_{i+4}, then (0+1)+(2+3) (sgemv kernel)
 * Each product x * (+-1/16) is exact, so the chains add +-x and the result is scaled by
 * 1/16 at the end (exact). Zeros are returned as +0 like the reference's accumulators.
 *
 * Also the butterfly order used for activations: radix-4 stages on base-4 digits
 * 0,1,2,3 (least significant first); b_i = ((a0+a1)+(a2+a3)) - 2*a_{3-i}.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fPIC -shared (no FMA contraction:
 * every add is an IEEE fp32 add, which is what the restatement means).
 */
#include <stdint.h>
#include <string.h>

static int h4neg(int a, int b) { return a + b == 3; }

static float sign_of(int j, int k) {
  int neg = 0;
  for (int d = 0; d < 4; ++d) neg ^= h4neg((j >> (2 * d)) & 3, (k >> (2 * d)) & 3);
  return neg ? -1.0f : 1.0f;
}

static float canon(float v) { return v == 0.0f ? 0.0f : v; }

/* S[k][j] = sign of H[j][k] (H is symmetric, so also of H[k][j]). */
static float S[256][256];
static int S_ready = 0;
static void init_signs(void) {
  if (S_ready) return;
  for (int k = 0; k < 256; ++k)
    for (int j = 0; j < 256; ++j) S[k][j] = sign_of(j, k);
  S_ready = 1;
}

static void rotate_group_reference(const float* x, float* y, int groups) {
  init_signs();
  if (groups >= 5) {
    float acc[256];
    for (int j = 0; j < 256; ++j) acc[j] = 0.0f;
    for (int k = 0; k < 256; ++k) {
      const float xk = x[k];
      for (int j = 0; j < 256; ++j) acc[j] = acc[j] + S[k][j] * xk;
    }
    for (int j = 0; j < 256; ++j) y[j] = canon(acc[j] * 0.0625f);
  } else if (groups >= 2) {
    static float lane[16][256];
    for (int l = 0; l < 16; ++l)
      for (int j = 0; j < 256; ++j) lane[l][j] = 0.0f;
    for (int t = 0; t < 16; ++t)
      for (int l = 0; l < 16; ++l) {
        const int k = 16 * t + l;
        const float xk = x[k];
        for (int j = 0; j < 256; ++j) lane[l][j] = lane[l][j] + S[k][j] * xk;
      }
    for (int w = 8; w >= 1; w >>= 1)
      for (int i = 0; i < w; ++i)
        for (int j = 0; j < 256; ++j) lane[i][j] = lane[2 * i][j] + lane[2 * i + 1][j];
    for (int j = 0; j < 256; ++j) y[j] = canon(lane[0][j] * 0.0625f);
  } else {
    static float lane[8][256];
    for (int l = 0; l < 8; ++l)
      for (int j = 0; j < 256; ++j) lane[l][j] = 0.0f;
    for (int t = 0; t < 32; ++t)
      for (int l = 0; l < 8; ++l) {
        const int k = 8 * t + l;
        const float xk = x[k];
        for (int j = 0; j < 256; ++j) lane[l][j] = lane[l][j] + S[k][j] * xk;
      }
    for (int j = 0; j < 256; ++j) {
      const float u0 = lane[0][j] + lane[4][j];
      const float u1 = lane[1][j] + lane[5][j];
      const float u2 = lane[2][j] + lane[6][j];
      const float u3 = lane[3][j] + lane[7][j];
      y[j] = canon(((u0 + u1) + (u2 + u3)) * 0.0625f);
    }
  }
}

/* x, out: fp32 [rows, K], K % 256 == 0. */
void oracle_rotate_reference(const float* x, int64_t rows, int64_t K, float* out) {
  const int groups = (int)(K / 256);
  for (int64_t r = 0; r < rows; ++r)
    for (int g = 0; g < groups; ++g)
      rotate_group_reference(x + r * K + 256 * g, out + r * K + 256 * g, groups);
}

static void bfly4(float* a0, float* a1, float* a2, float* a3) {
  const float s = (*a0 + *a1) + (*a2 + *a3);
  const float b0 = s - 2.0f * *a3;
  const float b1 = s - 2.0f * *a2;
  const float b2 = s - 2.0f * *a1;
  const float b3 = s - 2.0f * *a0;
  *a0 = b0; *a1 = b1; *a2 = b2; *a3 = b3;
}

void oracle_rotate_butterfly(const float* x, int64_t rows, int64_t K, float* out) {
  const int64_t groups = K / 256;
  float v[256];
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      memcpy(v, x + r * K + 256 * g, sizeof(v));
      for (int d = 0; d < 4; ++d) {
        const int stride = 1 << (2 * d);
        for (int base = 0; base < 256; ++base) {
          if ((base >> (2 * d)) & 3) continue; /* digit d of base must be 0 */
          bfly4(&v[base], &v[base + stride], &v[base + 2 * stride], &v[base + 3 * stride]);
        }
      }
      for (int j = 0; j < 256; ++j) out[r * K + 256 * g + j] = v[j] * 0.0625f;
    }
}
