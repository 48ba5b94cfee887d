// aex_oracle.cpp — TEST INFRASTRUCTURE ONLY: CPU restatement of the reference
// arithmetic for parity checks and the timed CPU baseline. See aex_oracle.h
// for the reference file:line each function follows and for how it is pinned.
#include "aex_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include <atomic>
#include <thread>

namespace {
// Parallel loop over [0, n) on all hardware threads (AEXO_THREADS overrides),
// dynamic chunks of `grain` iterations.
template <class F>
void parallel_for(int64_t n, int64_t grain, F&& fn) {
  int nt = static_cast<int>(std::thread::hardware_concurrency());
  if (const char* e = std::getenv("AEXO_THREADS")) nt = std::max(1, std::atoi(e));
  if (nt <= 1 || n <= grain) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  auto worker = [&] {
    while (true) {
      const int64_t b = next.fetch_add(grain);
      if (b >= n) break;
      const int64_t e = std::min(n, b + grain);
      for (int64_t i = b; i < e; ++i) fn(i);
    }
  };
  std::vector<std::thread> ts;
  for (int t = 1; t < nt; ++t) ts.emplace_back(worker);
  worker();
  for (auto& t : ts) t.join();
}
}  // namespace

extern "C" {

uint16_t aexo_f32_to_bf16(float v) {
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  const uint32_t rounded = bits + 0x7FFFu + ((bits >> 16) & 1u);  // wraps like Swift &+
  return static_cast<uint16_t>(rounded >> 16);
}

float aexo_bf16_to_f32(uint16_t u) {
  const uint32_t bits = static_cast<uint32_t>(u) << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

void aexo_f32_to_bf16_array(const float* x, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = aexo_f32_to_bf16(x[i]);
}

void aexo_bf16_to_f32_array(const uint16_t* x, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = aexo_bf16_to_f32(x[i]);
}

// volatile intermediates keep the compiler from contracting scale*q + bias
// into an FMA: the reference computes `scale * q + bias` in Swift Float, which
// rounds the product and then the sum.
static inline float mul_then_add(float s, float q, float b) {
  volatile float p = s * q;
  volatile float r = p + b;
  return r;
}

// One row of the dequant (DirectTEEncoder.embedRow, DirectTEEncoder.swift:104-123).
static void dequant_row(const uint32_t* packed_row, const uint16_t* scales_row, const uint16_t* biases_row, int k,
                        int group_size, uint16_t* out_row) {
  for (int g = 0; g < k / group_size; ++g) {
    const float scale = aexo_bf16_to_f32(scales_row[g]);
    const float bias = aexo_bf16_to_f32(biases_row[g]);
    const int col_base = g * group_size;
    for (int w = 0; w < group_size / 8; ++w) {
      const uint32_t p = packed_row[col_base / 8 + w];
      for (int nib = 0; nib < 8; ++nib) {
        const float q = static_cast<float>((p >> (4 * nib)) & 0xFu);
        out_row[col_base + w * 8 + nib] = aexo_f32_to_bf16(mul_then_add(scale, q, bias));
      }
    }
  }
}

void aexo_dequant_q4(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n, int k,
                     int group_size, uint16_t* out_bf16) {
  parallel_for(n, 64, [&](int64_t r) {
    dequant_row(packed + (size_t)r * (k / 8), scales + (size_t)r * (k / group_size),
                biases + (size_t)r * (k / group_size), k, group_size, out_bf16 + (size_t)r * k);
  });
}

void aexo_pack_q4(const uint8_t* codes, int n, int k, uint32_t* packed) {
  for (int r = 0; r < n; ++r)
    for (int w = 0; w < k / 8; ++w) {
      uint32_t p = 0;
      for (int nib = 0; nib < 8; ++nib) p |= static_cast<uint32_t>(codes[(size_t)r * k + w * 8 + nib] & 0xF) << (4 * nib);
      packed[(size_t)r * (k / 8) + w] = p;
    }
}

void aexo_qmm(const float* x, int m, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases,
              int n, int k, int group_size, float* y) {
  // Blocks of kRows weight rows: each block is dequantized once, then every x
  // row is read once per block (not once per weight row). The f64 dot products
  // are vectorized (a fixed lane order: deterministic for a given build).
  constexpr int kRows = 16;
  const int64_t blocks = (n + kRows - 1) / kRows;
  parallel_for(blocks, 1, [&](int64_t blk) {
    const int r0 = static_cast<int>(blk * kRows);
    const int nr = std::min(kRows, n - r0);
    std::vector<uint16_t> wrow_bf(k);
    std::vector<float> wblk(static_cast<size_t>(nr) * k);
    for (int j = 0; j < nr; ++j) {
      const size_t r = static_cast<size_t>(r0 + j);
      dequant_row(packed + r * (k / 8), scales + r * (k / group_size), biases + r * (k / group_size), k, group_size,
                  wrow_bf.data());
      for (int c = 0; c < k; ++c) wblk[(size_t)j * k + c] = aexo_bf16_to_f32(wrow_bf[c]);
    }
    for (int i = 0; i < m; ++i) {
      const float* xi = x + (size_t)i * k;
      for (int j = 0; j < nr; ++j) {
        const float* w = wblk.data() + (size_t)j * k;
        double acc = 0.0;
#pragma omp simd reduction(+ : acc)
        for (int c = 0; c < k; ++c) acc += (double)xi[c] * (double)w[c];
        y[(size_t)i * n + r0 + j] = static_cast<float>(acc);
      }
    }
  });
}

void aexo_qmv(const float* x, int m, const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int n,
              int k, int group_size, float* y) {
  const int groups = k / group_size;
  parallel_for(n, 16, [&](int64_t r) {
    const uint32_t* pr = packed + (size_t)r * (k / 8);
    for (int i = 0; i < m; ++i) {
      const float* xi = x + (size_t)i * k;
      double acc = 0.0;
      for (int g = 0; g < groups; ++g) {
        double qdot = 0.0, xsum = 0.0;
        for (int c = g * group_size; c < (g + 1) * group_size; ++c) {
          const uint32_t q = (pr[c / 8] >> (4 * (c % 8))) & 0xFu;
          qdot += (double)xi[c] * (double)q;
          xsum += (double)xi[c];
        }
        acc += (double)aexo_bf16_to_f32(scales[(size_t)r * groups + g]) * qdot +
               (double)aexo_bf16_to_f32(biases[(size_t)r * groups + g]) * xsum;
      }
      y[(size_t)i * n + r] = static_cast<float>(acc);
    }
  });
}

void aexo_rope_freqs(const float* ids, int n, float theta, const int* axes_dim, int n_axes, float* cos_out,
                     float* sin_out) {
  int half_total = 0;
  for (int a = 0; a < n_axes; ++a) half_total += axes_dim[a] / 2;
  for (int r = 0; r < n; ++r) {
    int col = 0;
    for (int a = 0; a < n_axes; ++a) {
      const int dim = axes_dim[a];
      const float pos = ids[(size_t)r * n_axes + a];
      for (int i = 0; i < dim / 2; ++i) {
        const float sc = static_cast<float>(2 * i) / static_cast<float>(dim);
        const float omega = 1.0f / std::pow(theta, sc);
        const float angle = pos * omega;
        cos_out[(size_t)r * half_total + col] = std::cos(angle);
        sin_out[(size_t)r * half_total + col] = std::sin(angle);
        ++col;
      }
    }
  }
}

void aexo_grid_ids(int height, int width, float t_coord, float layer, float* ids_out) {
  size_t r = 0;
  for (int h = 0; h < height; ++h)
    for (int w = 0; w < width; ++w, ++r) {
      ids_out[r * 4 + 0] = t_coord;
      ids_out[r * 4 + 1] = static_cast<float>(h);
      ids_out[r * 4 + 2] = static_cast<float>(w);
      ids_out[r * 4 + 3] = layer;
    }
}

void aexo_text_ids(int length, float* ids_out) {
  for (int i = 0; i < length; ++i) {
    ids_out[(size_t)i * 4 + 0] = 0.f;
    ids_out[(size_t)i * 4 + 1] = 0.f;
    ids_out[(size_t)i * 4 + 2] = 0.f;
    ids_out[(size_t)i * 4 + 3] = static_cast<float>(i);
  }
}

void aexo_rmsnorm(const float* x, int rows, int d, const float* w, float eps, float* y) {
  parallel_for(rows, 256, [&](int64_t r) {
    const float* xr = x + (size_t)r * d;
    double ss = 0.0;
    for (int i = 0; i < d; ++i) ss += (double)xr[i] * xr[i];
    const float inv = static_cast<float>(1.0 / std::sqrt(ss / d + (double)eps));
    for (int i = 0; i < d; ++i) y[(size_t)r * d + i] = xr[i] * inv * (w ? w[i] : 1.0f);
  });
}

void aexo_rope_apply(float* x, int s, int h, int d, const float* cos_t, const float* sin_t) {
  const int half = d / 2;
  parallel_for(s, 64, [&](int64_t t) {
    for (int hh = 0; hh < h; ++hh) {
      float* row = x + ((size_t)t * h + hh) * d;
      for (int i = 0; i < half; ++i) {
        const float c = cos_t[(size_t)t * half + i], sn = sin_t[(size_t)t * half + i];
        const float re = row[2 * i], im = row[2 * i + 1];
        row[2 * i] = re * c + (-im) * sn;
        row[2 * i + 1] = im * c + re * sn;
      }
    }
  });
}

void aexo_sdpa(const float* q, const float* k, const float* v, float* out, int b, int s, int h, int d,
               int64_t stride_b, int64_t stride_s, int64_t stride_h, float scale, int q_begin, int q_end) {
  q_begin = std::max(0, q_begin);
  q_end = std::min(s, q_end);
  if (q_end <= q_begin) return;
  // Blocks of kQB query rows share every key/value row while it is in cache.
  constexpr int kQB = 32;
  const int nq = q_end - q_begin;
  const int nblk = (nq + kQB - 1) / kQB;
  const int64_t total = (int64_t)b * h * nblk;
  parallel_for(total, 1, [&](int64_t job) {
    thread_local std::vector<float> sc, acc;
    sc.resize((size_t)kQB * s);
    acc.resize((size_t)kQB * d);
    const int blk = static_cast<int>(job % nblk);
    const int hh = static_cast<int>((job / nblk) % h);
    const int bb = static_cast<int>(job / ((int64_t)nblk * h));
    const int i0 = q_begin + blk * kQB;
    const int nb = std::min(kQB, q_end - i0);
    const float* qrow[kQB];
    for (int i = 0; i < nb; ++i) qrow[i] = q + bb * stride_b + (int64_t)(i0 + i) * stride_s + hh * stride_h;
    for (int j = 0; j < s; ++j) {
      const float* kr = k + bb * stride_b + (int64_t)j * stride_s + hh * stride_h;
      for (int i = 0; i < nb; ++i) {
        const float* qr = qrow[i];
        float dot = 0.f;
#pragma omp simd reduction(+ : dot)
        for (int t = 0; t < d; ++t) dot += qr[t] * kr[t];
        sc[(size_t)i * s + j] = dot * scale;
      }
    }
    double l[kQB];
    for (int i = 0; i < nb; ++i) {
      float* row = &sc[(size_t)i * s];
      float mx = -INFINITY;
      for (int j = 0; j < s; ++j) mx = std::max(mx, row[j]);
      double sum = 0.0;
      for (int j = 0; j < s; ++j) {
        row[j] = std::exp(row[j] - mx);
        sum += row[j];
      }
      l[i] = sum;
    }
    std::fill(acc.begin(), acc.end(), 0.f);
    for (int j = 0; j < s; ++j) {
      const float* vr = v + bb * stride_b + (int64_t)j * stride_s + hh * stride_h;
      for (int i = 0; i < nb; ++i) {
        const float pij = sc[(size_t)i * s + j];
        float* a = &acc[(size_t)i * d];
#pragma omp simd
        for (int t = 0; t < d; ++t) a[t] += pij * vr[t];
      }
    }
    for (int i = 0; i < nb; ++i) {
      float* orow = out + bb * stride_b + (int64_t)(i0 + i) * stride_s + hh * stride_h;
      for (int t = 0; t < d; ++t) orow[t] = static_cast<float>(acc[(size_t)i * d + t] / l[i]);
    }
  });
}

void aexo_joint_attention(const float* q, const float* k, const float* v, float* out, int b, int s, int h, int d,
                          const float* norm_q_w, const float* norm_k_w, float eps, const float* cos_t,
                          const float* sin_t, float scale, int q_begin, int q_end) {
  const size_t per_batch = (size_t)s * h * d;
  std::vector<float> qn(q, q + per_batch * b), kn(k, k + per_batch * b);
  if (norm_q_w) aexo_rmsnorm(qn.data(), b * s * h, d, norm_q_w, eps, qn.data());
  if (norm_k_w) aexo_rmsnorm(kn.data(), b * s * h, d, norm_k_w, eps, kn.data());
  if (cos_t && sin_t)
    for (int bb = 0; bb < b; ++bb) {
      aexo_rope_apply(qn.data() + bb * per_batch, s, h, d, cos_t, sin_t);
      aexo_rope_apply(kn.data() + bb * per_batch, s, h, d, cos_t, sin_t);
    }
  aexo_sdpa(qn.data(), kn.data(), v, out, b, s, h, d, (int64_t)per_batch, (int64_t)h * d, d, scale, q_begin,
            q_end);
}

float aexo_linear_mu(int image_seq_len, int base_seq_len, int max_seq_len, float base_shift, float max_shift) {
  const float m = (max_shift - base_shift) / static_cast<float>(max_seq_len - base_seq_len);
  const float bb = base_shift - m * static_cast<float>(base_seq_len);
  return m * static_cast<float>(image_seq_len) + bb;
}

float aexo_time_shift(float mu, float t, float sigma_power) {
  const float e = std::exp(mu);
  const float inv = std::pow(1.0f / t - 1.0f, sigma_power);
  return e / (e + inv);
}

void aexo_schedule(int steps, int image_seq_len, float* sigmas, float* timesteps) {
  const float mu = aexo_linear_mu(image_seq_len, 256, 4096, 0.5f, 1.15f);
  for (int i = 0; i < steps; ++i) {
    float base;
    if (steps == 1) {
      base = 1.0f;
    } else {
      const float t = static_cast<float>(i) / static_cast<float>(steps - 1);
      const float end = 1.0f / static_cast<float>(steps);
      base = 1.0f + (end - 1.0f) * t;
    }
    const float sh = aexo_time_shift(mu, base, 1.0f);
    sigmas[i] = sh;
    timesteps[i] = sh * 1000.0f;
  }
  sigmas[steps] = 0.0f;
}

void aexo_timestep_embedding(const float* t, int n, int dim, float* out) {
  const int half = dim / 2;
  const float log10000 = std::log(10000.0f);
  std::vector<float> freqs(half);
  for (int i = 0; i < half; ++i) freqs[i] = std::exp(-log10000 * static_cast<float>(i) / static_cast<float>(half));
  for (int r = 0; r < n; ++r) {
    float* o = out + (size_t)r * dim;
    for (int i = 0; i < half; ++i) {
      const float arg = t[r] * freqs[i];
      o[i] = std::cos(arg);
      o[half + i] = std::sin(arg);
    }
    if (dim % 2 == 1) o[dim - 1] = 0.f;
  }
}

void aexo_ln_mod(const float* x, int rows, int d, const float* scale, const float* shift, float eps, float* y) {
  parallel_for(rows, 64, [&](int64_t r) {
    const float* xr = x + (size_t)r * d;
    double s1 = 0.0, s2 = 0.0;
    for (int i = 0; i < d; ++i) {
      s1 += xr[i];
      s2 += (double)xr[i] * xr[i];
    }
    const double mean = s1 / d;
    const double var = s2 / d - mean * mean;
    const float inv = static_cast<float>(1.0 / std::sqrt(var + (double)eps));
    for (int i = 0; i < d; ++i) {
      const float nrm = (xr[i] - static_cast<float>(mean)) * inv;
      y[(size_t)r * d + i] = (scale[i] + 1.0f) * nrm + shift[i];
    }
  });
}

void aexo_swiglu(const float* g, const float* u, size_t n, float* y) {
  for (size_t i = 0; i < n; ++i) y[i] = g[i] / (1.0f + std::exp(-g[i])) * u[i];
}

void aexo_gate_add(const float* x, const float* gate, const float* v, int rows, int d, float* y) {
  for (int r = 0; r < rows; ++r)
    for (int i = 0; i < d; ++i) y[(size_t)r * d + i] = x[(size_t)r * d + i] + gate[i] * v[(size_t)r * d + i];
}

}  // extern "C"
