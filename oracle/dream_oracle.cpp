// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
//
// CPU restatement of the reference runtime's arithmetic for the hot path
// (heellowdsf/DreamCompiler, paths relative to the project root). Only the
// tests, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
// load this library, and only as the checker or the timed CPU baseline; the
// product path (libdgx / libdream_b200) never links or calls it.
//
// Pinned against the reference itself: tests/golden/ holds vectors produced by
// the reference runtime compiled from its own sources (oracle/build_ref.sh ->
// oracle/_ref/libdream_ref.so, tests/golden/make_golden.py), and
// tests/test_oracle.py checks every function below against them.
//
// Every function is extern "C" with plain pointers so Python (ctypes) and C
// harnesses can call it. Loops that the reference parallelises with OpenMP
// are parallelised the same way; the rest are plain loops.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>

extern "C" {

// ---------------------------------------------------------------- bf16
// fp32 -> bf16 -> fp32 with round-to-nearest-even on the raw bits, as
// dream_to_bf16 (runtime/nn/training.inc:1969-1976).
float orc_to_bf16(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  b += 0x7FFFu + ((b >> 16) & 1u);
  b &= 0xFFFF0000u;
  float r;
  std::memcpy(&r, &b, 4);
  return r;
}
void orc_round_bf16(const float* in, float* out, long n) {
  for (long i = 0; i < n; ++i) out[i] = orc_to_bf16(in[i]);
}
// Same rounding, but emitting the 16-bit patterns (what a bf16 buffer holds).
void orc_bf16_bits(const float* in, uint16_t* out, long n) {
  for (long i = 0; i < n; ++i) {
    float r = orc_to_bf16(in[i]);
    uint32_t b;
    std::memcpy(&b, &r, 4);
    out[i] = (uint16_t)(b >> 16);
  }
}

// ---------------------------------------------------------------- GEMM
// C = A.B in double, row-major, as dream_gemm_d (runtime/ops/elementwise.inc:
// 593-638) and its naive check gemm_ref_d (:876-886). Summation order is
// k-ascending per output; OpenMP over rows.
void orc_gemm_f64(const double* A, const double* B, double* C, int M, int K, int N) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i) {
    double* c = C + (size_t)i * N;
    for (int j = 0; j < N; ++j) c[j] = 0.0;
    for (int k = 0; k < K; ++k) {
      const double a = A[(size_t)i * K + k];
      const double* b = B + (size_t)k * N;
      for (int j = 0; j < N; ++j) c[j] += a * b[j];
    }
  }
}

// Same, for a subset of rows: C[r,:] = A[rows[r],:].B (used to verify large
// GEMMs on a sample of rows).
void orc_gemm_rows_f64(const double* A, const double* B, double* C, const int* rows, int nrows, int K, int N) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < nrows; ++r) {
    double* c = C + (size_t)r * N;
    for (int j = 0; j < N; ++j) c[j] = 0.0;
    const double* a = A + (size_t)rows[r] * K;
    for (int k = 0; k < K; ++k) {
      const double* b = B + (size_t)k * N;
      for (int j = 0; j < N; ++j) c[j] += a[k] * b[j];
    }
  }
}

// fp32-accumulated GEMM: the f32-mirror path of tensor_matmul
// (dream_gemm_f32, runtime/ops/elementwise.inc:689-738). The reference blocks
// K in chunks of KC=256 and adds each chunk's fp32 partial sum into C; this
// restatement keeps that two-level order (chunk partials, then chunk sum).
void orc_gemm_f32(const float* A, const float* B, float* C, int M, int K, int N) {
  const int KC = 256;
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i) {
    std::vector<float> part((size_t)N);
    float* c = C + (size_t)i * N;
    for (int j = 0; j < N; ++j) c[j] = 0.f;
    for (int k0 = 0; k0 < K; k0 += KC) {
      const int k1 = std::min(K, k0 + KC);
      std::fill(part.begin(), part.end(), 0.f);
      for (int k = k0; k < k1; ++k) {
        const float a = A[(size_t)i * K + k];
        const float* b = B + (size_t)k * N;
        for (int j = 0; j < N; ++j) part[j] = std::fma(a, b[j], part[j]);
      }
      for (int j = 0; j < N; ++j) c[j] += part[j];
    }
  }
}

// "matmul" backward (runtime/ops/autograd.inc:91-125): accumulates
//   dA[i,k] += sum_j dY[i,j]*B[k,j]     dB[k,j] += sum_i A[i,k]*dY[i,j]
// in double, into existing gradient buffers.
void orc_matmul_bwd(const double* A, const double* B, const double* dY, double* dA, double* dB, int M, int K,
                    int N) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i) {
    const double* dy = dY + (size_t)i * N;
    for (int k = 0; k < K; ++k) {
      const double* b = B + (size_t)k * N;
      double acc = 0.0;
      for (int j = 0; j < N; ++j) acc += dy[j] * b[j];
      dA[(size_t)i * K + k] += acc;
    }
  }
#pragma omp parallel for schedule(static)
  for (int k = 0; k < K; ++k) {
    double* db = dB + (size_t)k * N;
    for (int i = 0; i < M; ++i) {
      const double a = A[(size_t)i * K + k];
      const double* dy = dY + (size_t)i * N;
      for (int j = 0; j < N; ++j) db[j] += a * dy[j];
    }
  }
}

// dream_bmm (runtime/ops/elementwise.inc:1218-1252): per batch b,
// C_b[M,N] = A_b[M,K].B_b[K,N] in double, operands flat (batch, M*K) etc.
void orc_bmm_f64(const double* A, const double* B, double* C, int batch, int M, int K, int N) {
  for (int b = 0; b < batch; ++b)
    orc_gemm_f64(A + (size_t)b * M * K, B + (size_t)b * K * N, C + (size_t)b * M * N, M, K, N);
}

// "bmm" backward (runtime/ops/autograd.inc:549-574): per batch, the "matmul"
// backward accumulated into dA_b, dB_b.
void orc_bmm_bwd(const double* A, const double* B, const double* dC, double* dA, double* dB, int batch, int M,
                 int K, int N) {
  for (int b = 0; b < batch; ++b)
    orc_matmul_bwd(A + (size_t)b * M * K, B + (size_t)b * K * N, dC + (size_t)b * M * N, dA + (size_t)b * M * K,
                   dB + (size_t)b * K * N, M, K, N);
}

// dream_linear / dream_linear_relu (runtime/ops/elementwise.inc:1432-1521):
// Y[i,j] = b[j] + sum_k X[i,k]*W[j,k]  (W stored out x in), then ReLU.
void orc_linear(const double* X, const double* W, const double* b, double* Y, int N, int in_dim, int out_dim,
                int relu) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i)
    for (int j = 0; j < out_dim; ++j) {
      double s = b ? b[j] : 0.0;
      for (int k = 0; k < in_dim; ++k) s += X[(size_t)i * in_dim + k] * W[(size_t)j * in_dim + k];
      Y[(size_t)i * out_dim + j] = (relu && s < 0) ? 0.0 : s;
    }
}

// linear backward (runtime/ops/autograd.inc:156-211): with g = dY masked by
// Y>0 for linear_relu, db[j] += sum_i g[i,j]; dX[i,k] += sum_j g[i,j]*W[j,k];
// dW[j,k] += sum_i g[i,j]*X[i,k].
void orc_linear_bwd(const double* X, const double* W, const double* Y, const double* dY, double* dX, double* dW,
                    double* db, int N, int in_dim, int out_dim, int relu) {
  std::vector<double> g((size_t)N * out_dim);
  for (size_t t = 0; t < g.size(); ++t) g[t] = (relu && Y[t] <= 0.0) ? 0.0 : dY[t];
  if (db)
    for (int j = 0; j < out_dim; ++j) {
      double s = 0;
      for (int i = 0; i < N; ++i) s += g[(size_t)i * out_dim + j];
      db[j] += s;
    }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i)
    for (int k = 0; k < in_dim; ++k) {
      double s = 0;
      for (int j = 0; j < out_dim; ++j) s += g[(size_t)i * out_dim + j] * W[(size_t)j * in_dim + k];
      dX[(size_t)i * in_dim + k] += s;
    }
#pragma omp parallel for schedule(static)
  for (int j = 0; j < out_dim; ++j)
    for (int k = 0; k < in_dim; ++k) {
      double s = 0;
      for (int i = 0; i < N; ++i) s += g[(size_t)i * out_dim + j] * X[(size_t)i * in_dim + k];
      dW[(size_t)j * in_dim + k] += s;
    }
}

// ---------------------------------------------------------------- attention
// Causal FlashAttention forward, f64, as dream_flash_attention's CPU loop
// (runtime/nn/training.inc:366-399): per query row i, K/V blocks of Bc keys
// (j <= i), running max m, normaliser l and accumulator, O_i = acc / l.
// Layout [B][S][dk]. Also emits the natural-log LSE m + log(l) per row, which
// the reference does not store but which is what the device kernel saves.
void orc_flash_fwd(const double* Q, const double* K, const double* V, double* O, double* lse, int B, int S,
                   int dk, int Bc) {
  if (Bc < 1) Bc = 64;
  const double scale = 1.0 / std::sqrt((double)dk);
#pragma omp parallel for schedule(dynamic)
  for (int b = 0; b < B; ++b) {
    const double* Qb = Q + (size_t)b * S * dk;
    const double* Kb = K + (size_t)b * S * dk;
    const double* Vb = V + (size_t)b * S * dk;
    double* Ob = O + (size_t)b * S * dk;
    std::vector<double> sc((size_t)Bc), acc((size_t)dk);
    for (int i = 0; i < S; ++i) {
      double m = -1e30, l = 0.0;
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int jb = 0; jb <= i; jb += Bc) {
        const int je = std::min(i, jb + Bc - 1);
        double mb = -1e30;
        for (int j = jb; j <= je; ++j) {
          double s = 0;
          for (int k = 0; k < dk; ++k) s += Qb[(size_t)i * dk + k] * Kb[(size_t)j * dk + k];
          sc[j - jb] = s * scale;
          mb = std::max(mb, sc[j - jb]);
        }
        const double mn = std::max(m, mb), corr = std::exp(m - mn);
        l *= corr;
        for (int k = 0; k < dk; ++k) acc[k] *= corr;
        for (int j = jb; j <= je; ++j) {
          const double p = std::exp(sc[j - jb] - mn);
          l += p;
          for (int k = 0; k < dk; ++k) acc[k] += p * Vb[(size_t)j * dk + k];
        }
        m = mn;
      }
      const double inv = l > 0.0 ? 1.0 / l : 0.0;
      for (int k = 0; k < dk; ++k) Ob[(size_t)i * dk + k] = acc[k] * inv;
      if (lse) lse[(size_t)b * S + i] = m + std::log(l);
    }
  }
}

// Causal FlashAttention backward, f64, as the "flash_attention" branch of
// backward() (runtime/ops/autograd.inc:779-840): pass 1 recomputes each row's
// (m, l) over blocks of 64 keys, pass 2 forms D_i = dO_i . O_i with O_i
// recomputed, pass 3 recomputes P_ij = exp(s_ij - m_i)/l_i and accumulates
// dV_j += P_ij dO_i, dQ_i += dS_ij K_j scale, dK_j += dS_ij Q_i scale with
// dS_ij = P_ij (dO_i.V_j - D_i). Gradients are ADDED into dQ, dK, dV.
void orc_flash_bwd(const double* Q, const double* K, const double* V, const double* dO, double* dQ, double* dK,
                   double* dV, int B, int S, int dk) {
  const double scale = 1.0 / std::sqrt((double)dk);
  const int Bc = 64;
#pragma omp parallel for schedule(dynamic)
  for (int b = 0; b < B; ++b) {
    const double* Qb = Q + (size_t)b * S * dk;
    const double* Kb = K + (size_t)b * S * dk;
    const double* Vb = V + (size_t)b * S * dk;
    const double* dOb = dO + (size_t)b * S * dk;
    double* dQb = dQ + (size_t)b * S * dk;
    double* dKb = dK + (size_t)b * S * dk;
    double* dVb = dV + (size_t)b * S * dk;
    std::vector<double> row_m((size_t)S), row_l((size_t)S), Drow((size_t)S), sc((size_t)Bc), acc((size_t)dk);
    auto dot_qk = [&](int i, int j) {
      double s = 0;
      for (int k = 0; k < dk; ++k) s += Qb[(size_t)i * dk + k] * Kb[(size_t)j * dk + k];
      return s;
    };
    for (int i = 0; i < S; ++i) {
      double m = -1e30, l = 0.0;
      for (int jb = 0; jb <= i; jb += Bc) {
        const int je = std::min(i, jb + Bc - 1);
        double mb = -1e30;
        for (int j = jb; j <= je; ++j) {
          sc[j - jb] = dot_qk(i, j) * scale;
          mb = std::max(mb, sc[j - jb]);
        }
        const double mn = std::max(m, mb);
        l *= std::exp(m - mn);
        for (int j = jb; j <= je; ++j) l += std::exp(sc[j - jb] - mn);
        m = mn;
      }
      row_m[i] = m;
      row_l[i] = l;
    }
    for (int i = 0; i < S; ++i) {
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int j = 0; j <= i; ++j) {
        const double p = std::exp(dot_qk(i, j) * scale - row_m[i]) / row_l[i];
        for (int k = 0; k < dk; ++k) acc[k] += p * Vb[(size_t)j * dk + k];
      }
      double d = 0;
      for (int k = 0; k < dk; ++k) d += dOb[(size_t)i * dk + k] * acc[k];
      Drow[i] = d;
    }
    for (int i = 0; i < S; ++i) {
      for (int j = 0; j <= i; ++j) {
        const double p = std::exp(dot_qk(i, j) * scale - row_m[i]) / row_l[i];
        double dp = 0;
        for (int k = 0; k < dk; ++k) dp += dOb[(size_t)i * dk + k] * Vb[(size_t)j * dk + k];
        const double ds = p * (dp - Drow[i]);
        for (int k = 0; k < dk; ++k) {
          dVb[(size_t)j * dk + k] += p * dOb[(size_t)i * dk + k];
          dQb[(size_t)i * dk + k] += ds * Kb[(size_t)j * dk + k] * scale;
          dKb[(size_t)j * dk + k] += ds * Qb[(size_t)i * dk + k] * scale;
        }
      }
    }
  }
}

// Materialised causal SDPA (dream_attention_causal, runtime/nn/training.inc:
// 225-263): the reference FlashAttention is tested against. causal=0 gives
// dream_attention (:178-220).
void orc_attention(const double* Q, const double* K, const double* V, double* O, int B, int S, int dk,
                   int causal) {
  const double scale = 1.0 / std::sqrt((double)dk);
#pragma omp parallel for schedule(dynamic)
  for (int b = 0; b < B; ++b) {
    const double* Qb = Q + (size_t)b * S * dk;
    const double* Kb = K + (size_t)b * S * dk;
    const double* Vb = V + (size_t)b * S * dk;
    double* Ob = O + (size_t)b * S * dk;
    std::vector<double> a((size_t)S);
    for (int i = 0; i < S; ++i) {
      const int jmax = causal ? i : S - 1;
      double mx = -1e30;
      for (int j = 0; j <= jmax; ++j) {
        double s = 0;
        for (int k = 0; k < dk; ++k) s += Qb[(size_t)i * dk + k] * Kb[(size_t)j * dk + k];
        a[j] = s * scale;
        mx = std::max(mx, a[j]);
      }
      double sum = 0;
      for (int j = 0; j <= jmax; ++j) {
        a[j] = std::exp(a[j] - mx);
        sum += a[j];
      }
      for (int k = 0; k < dk; ++k) {
        double s = 0;
        for (int j = 0; j <= jmax; ++j) s += a[j] / sum * Vb[(size_t)j * dk + k];
        Ob[(size_t)i * dk + k] = s;
      }
    }
  }
}

// Backward of the materialised SDPA ("attention" and "attention_causal"
// branches, runtime/ops/autograd.inc:675-778): recompute A = softmax(QK^T*sc)
// (masked to j <= i when causal), then dV += A^T dO, dA = dO V^T,
// dS = A o (dA - rowsum(dA o A)), dQ += dS K sc, dK += dS^T Q sc.
void orc_attention_bwd(const double* Q, const double* K, const double* V, const double* dO, double* dQ, double* dK,
                       double* dV, int B, int S, int dk, int causal) {
  const double scale = 1.0 / std::sqrt((double)dk);
#pragma omp parallel for schedule(dynamic)
  for (int b = 0; b < B; ++b) {
    const size_t o = (size_t)b * S * dk;
    const double *Qb = Q + o, *Kb = K + o, *Vb = V + o, *dOb = dO + o;
    double *dQb = dQ + o, *dKb = dK + o, *dVb = dV + o;
    std::vector<double> A((size_t)S * S, 0.0), dS((size_t)S * S, 0.0);
    for (int i = 0; i < S; ++i) {
      const int jmax = causal ? i : S - 1;
      double mx = -1e300;
      for (int j = 0; j <= jmax; ++j) {
        double s = 0;
        for (int k = 0; k < dk; ++k) s += Qb[(size_t)i * dk + k] * Kb[(size_t)j * dk + k];
        A[(size_t)i * S + j] = s * scale;
        mx = std::max(mx, A[(size_t)i * S + j]);
      }
      double sum = 0;
      for (int j = 0; j <= jmax; ++j) sum += (A[(size_t)i * S + j] = std::exp(A[(size_t)i * S + j] - mx));
      for (int j = 0; j <= jmax; ++j) A[(size_t)i * S + j] /= sum;
      // dA_ij = dO_i . V_j and the row term sum_j dA_ij A_ij
      double rd = 0;
      for (int j = 0; j <= jmax; ++j) {
        double s = 0;
        for (int k = 0; k < dk; ++k) s += dOb[(size_t)i * dk + k] * Vb[(size_t)j * dk + k];
        dS[(size_t)i * S + j] = s;
        rd += s * A[(size_t)i * S + j];
      }
      for (int j = 0; j <= jmax; ++j) dS[(size_t)i * S + j] = A[(size_t)i * S + j] * (dS[(size_t)i * S + j] - rd);
    }
    for (int j = 0; j < S; ++j)
      for (int k = 0; k < dk; ++k) {
        double sv = 0, sk = 0;
        for (int i = 0; i < S; ++i) {
          sv += A[(size_t)i * S + j] * dOb[(size_t)i * dk + k];
          sk += dS[(size_t)i * S + j] * Qb[(size_t)i * dk + k];
        }
        dVb[(size_t)j * dk + k] += sv;
        dKb[(size_t)j * dk + k] += sk * scale;
      }
    for (int i = 0; i < S; ++i)
      for (int k = 0; k < dk; ++k) {
        double s = 0;
        for (int j = 0; j < S; ++j) s += dS[(size_t)i * S + j] * Kb[(size_t)j * dk + k];
        dQb[(size_t)i * dk + k] += s * scale;
      }
  }
}

// ---------------------------------------------------------------- convolution
// dream_conv2d / dream_conv2d_padded (runtime/nn/conv.inc:12-187): per
// sample, col = im2col(zero-padded input, stride) [Cin*KH*KW][OH*OW]
// (runtime/nn/im2col.inc:2-13, conv.inc:151-163), Y_n = K . col (f64),
// then + bias[co] on every position of channel co.
static void orc_im2col(const double* x, double* col, int Cin, int H, int W, int KH, int KW, int pad, int stride,
                       int OH, int OW) {
  int r = 0;
  for (int ci = 0; ci < Cin; ++ci)
    for (int kh = 0; kh < KH; ++kh)
      for (int kw = 0; kw < KW; ++kw, ++r)
        for (int oh = 0; oh < OH; ++oh)
          for (int ow = 0; ow < OW; ++ow) {
            const int h = oh * stride - pad + kh, w = ow * stride - pad + kw;
            col[(size_t)r * OH * OW + oh * OW + ow] =
                (h >= 0 && h < H && w >= 0 && w < W) ? x[((size_t)ci * H + h) * W + w] : 0.0;
          }
}

void orc_conv2d_fwd(const double* X, const double* K, const double* bias, double* Y, int N, int Cin, int H, int W,
                    int Cout, int KH, int KW, int pad, int stride) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  const int ckk = Cin * KH * KW, ohw = OH * OW;
#pragma omp parallel for schedule(dynamic)
  for (int n = 0; n < N; ++n) {
    std::vector<double> col((size_t)ckk * ohw);
    orc_im2col(X + (size_t)n * Cin * H * W, col.data(), Cin, H, W, KH, KW, pad, stride, OH, OW);
    double* y = Y + (size_t)n * Cout * ohw;
    orc_gemm_f64(K, col.data(), y, Cout, ckk, ohw);
    if (bias)
      for (int co = 0; co < Cout; ++co)
        for (int j = 0; j < ohw; ++j) y[(size_t)co * ohw + j] += bias[co];
  }
}

// "conv2d" backward (runtime/ops/autograd.inc:507-535), accumulating:
// dK[co][r] += sum_j dY_n[co][j] col_n[r][j]; dX_n += col2im(K^T . dY_n)
// (runtime/nn/im2col.inc:14-25), with the forward's pad / stride geometry.
void orc_conv2d_bwd(const double* X, const double* K, const double* dY, double* dX, double* dK, int N, int Cin,
                    int H, int W, int Cout, int KH, int KW, int pad, int stride) {
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  const int ckk = Cin * KH * KW, ohw = OH * OW;
  std::vector<double> col((size_t)ckk * ohw), dcol((size_t)ckk * ohw);
  for (int n = 0; n < N; ++n) {
    const double* go = dY + (size_t)n * Cout * ohw;
    orc_im2col(X + (size_t)n * Cin * H * W, col.data(), Cin, H, W, KH, KW, pad, stride, OH, OW);
#pragma omp parallel for schedule(static)
    for (int co = 0; co < Cout; ++co)
      for (int r = 0; r < ckk; ++r) {
        double s = 0;
        for (int j = 0; j < ohw; ++j) s += go[(size_t)co * ohw + j] * col[(size_t)r * ohw + j];
        dK[(size_t)co * ckk + r] += s;
      }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < ckk; ++r)
      for (int j = 0; j < ohw; ++j) {
        double s = 0;
        for (int co = 0; co < Cout; ++co) s += K[(size_t)co * ckk + r] * go[(size_t)co * ohw + j];
        dcol[(size_t)r * ohw + j] = s;
      }
    double* dx = dX + (size_t)n * Cin * H * W;
    int r = 0;
    for (int ci = 0; ci < Cin; ++ci)
      for (int kh = 0; kh < KH; ++kh)
        for (int kw = 0; kw < KW; ++kw, ++r)
          for (int oh = 0; oh < OH; ++oh)
            for (int ow = 0; ow < OW; ++ow) {
              const int h = oh * stride - pad + kh, w = ow * stride - pad + kw;
              if (h >= 0 && h < H && w >= 0 && w < W) dx[((size_t)ci * H + h) * W + w] += dcol[(size_t)r * ohw + oh * OW + ow];
            }
  }
}

// ---------------------------------------------------------------- int8
// Per-tensor symmetric quantiser of export_c_header_int8
// (runtime/nn/training.inc:3668-3692): scale = max|w|/127 (1 if ~0),
// q = clamp(lround(clamp(w/scale, -128, 127)), -128, 127).
void orc_quantize_per_tensor(const double* w, long n, int8_t* q, double* scale_out) {
  double mx = 0;
  for (long i = 0; i < n; ++i) mx = std::max(mx, std::fabs(w[i]));
  const double scale = mx > 1e-30 ? mx / 127.0 : 1.0;
  for (long i = 0; i < n; ++i) {
    double v = w[i] / scale;
    v = std::min(127.0, std::max(-128.0, v));
    long r = std::lround(v);
    r = std::min(127L, std::max(-128L, r));
    q[i] = (int8_t)r;
  }
  *scale_out = scale;
}

// The emitted dense_q (runtime/nn/training.inc:3738-3752) generalised to a
// per-output-channel scale and a batch of rows:
//   acc = b[j]; for k: acc += scale[j] * (float)w[j,k] * x[k]   (fp32, k ascending)
void orc_dense_q(const float* X, const int8_t* W, const float* scale, const float* bias, float* Y, int B, int N,
                 int K) {
#pragma omp parallel for schedule(static)
  for (int b = 0; b < B; ++b)
    for (int j = 0; j < N; ++j) {
      float acc = bias ? bias[j] : 0.f;
      const int8_t* wr = W + (size_t)j * K;
      const float* x = X + (size_t)b * K;
      for (int k = 0; k < K; ++k) acc += scale[j] * ((float)wr[k]) * x[k];
      Y[(size_t)b * N + j] = acc;
    }
}

// Exact integer core of the W8A8 mode: acc[b,n] = sum_k Xq[b,k]*W[n,k].
void orc_i8_gemm(const int8_t* Xq, const int8_t* W, int32_t* acc, int B, int N, int K) {
#pragma omp parallel for schedule(static)
  for (int b = 0; b < B; ++b)
    for (int n = 0; n < N; ++n) {
      int64_t s = 0;
      for (int k = 0; k < K; ++k) s += (int64_t)Xq[(size_t)b * K + k] * (int64_t)W[(size_t)n * K + k];
      acc[(size_t)b * N + n] = (int32_t)s;
    }
}

// Per-row activation quantiser of the W8A8 mode: sx = max|x|/127 (1 if 0),
// q = clamp(round-half-away(x/sx), -127, 127), computed in fp32.
void orc_quantize_rows(const float* X, int8_t* Xq, float* sx, int B, int K) {
  for (int b = 0; b < B; ++b) {
    float mx = 0.f;
    for (int k = 0; k < K; ++k) mx = std::max(mx, std::fabs(X[(size_t)b * K + k]));
    const float s = mx > 0.f ? mx / 127.f : 1.f;
    sx[b] = s;
    const float inv = 1.f / s;
    for (int k = 0; k < K; ++k) {
      float v = std::round(X[(size_t)b * K + k] * inv);
      v = std::min(127.f, std::max(-127.f, v));
      Xq[(size_t)b * K + k] = (int8_t)v;
    }
  }
}

// ---------------------------------------------------------------- tensor parallel
// Shard widths of dream_tp_matmul_column (runtime/nn/training.inc:1604-1630):
// base = N/G, the first N%G shards get one extra column.
void orc_tp_shard(int N, int G, int g, int* col0, int* ncol) {
  const int base = N / G, rem = N % G;
  *ncol = base + (g < rem ? 1 : 0);
  *col0 = g * base + std::min(g, rem);
}
// Column-parallel matmul: Y[:, shard g] = X . W[:, shard g] for every g, the
// shards placed side by side ("all-gather"), each shard an f64 GEMM.
void orc_tp_matmul_column(const double* X, const double* W, double* Y, int M, int K, int N, int G) {
  if (G < 1) G = 1;
  for (int g = 0; g < G; ++g) {
    int c0, nc;
    orc_tp_shard(N, G, g, &c0, &nc);
    if (nc <= 0) continue;
    std::vector<double> Wg((size_t)K * nc), Yg((size_t)M * nc);
    for (int k = 0; k < K; ++k)
      for (int c = 0; c < nc; ++c) Wg[(size_t)k * nc + c] = W[(size_t)k * N + c0 + c];
    orc_gemm_f64(X, Wg.data(), Yg.data(), M, K, nc);
    for (int i = 0; i < M; ++i)
      for (int c = 0; c < nc; ++c) Y[(size_t)i * N + c0 + c] = Yg[(size_t)i * nc + c];
  }
}

}  // extern "C"
