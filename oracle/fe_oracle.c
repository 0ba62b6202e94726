/* CPU restatement of the reference optimizer hot path.
 *
 * TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.  See
 * fe_oracle.h for the contract and the reference routine each function
 * restates.  Compiled with -ffp-contract=off so that float expressions round
 * exactly as written, like the reference's -O2 x86-64 build.
 */
#define _GNU_SOURCE
#include "fe_oracle.h"

#include <float.h>
#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* t-SNE: grid size policy                                             */
/* ------------------------------------------------------------------ */

/* env_positive_int + tsne_fft_grid_size, src/tsne_neighbors.cpp:282-291, 392-398. */
int or_tsne_grid_size(int n, int grid_override) {
  const int fallback = n >= 50000 ? 256 : (n >= 10000 ? 128 : 64);
  int requested = fallback;
  if (grid_override > 0) {
    requested = grid_override;
  } else {
    const char* raw = getenv("FASTEMBEDR_TSNE_FFT_GRID");
    if (raw != NULL && raw[0] != '\0') {
      char* end = NULL;
      const long parsed = strtol(raw, &end, 10);
      if (end != raw && parsed > 0L && parsed <= (long)INT_MAX) requested = (int)parsed;
    }
  }
  int grid = 32;
  while (grid < requested && grid < 512) grid <<= 1;
  if (grid < 32) grid = 32;
  if (grid > 512) grid = 512;
  return grid;
}

/* ------------------------------------------------------------------ */
/* t-SNE: affinities                                                   */
/* ------------------------------------------------------------------ */

void or_tsne_row_probabilities(const float* d, int k, double perplexity, float* p) {
  for (int j = 0; j < k; ++j) p[j] = 0.0f;
  int found = 0;
  float beta = 1.0f;
  float min_beta = -FLT_MAX;
  float max_beta = FLT_MAX;
  const float tol = 1e-5f;
  float sum_p = FLT_MIN;
  const float log_perp = (float)log(perplexity);
  for (int iter = 0; !found && iter < 200; ++iter) {
    sum_p = FLT_MIN;
    for (int j = 0; j < k; ++j) {
      const float dj = d[j];
      const float d2 = dj * dj;
      const float pj = expf(-beta * d2);
      p[j] = pj;
      sum_p += pj;
    }
    float entropy = 0.0f;
    for (int j = 0; j < k; ++j) {
      const float dj = d[j];
      entropy += beta * (dj * dj * p[j]);
    }
    entropy = entropy / sum_p + logf(sum_p);
    const float diff = entropy - log_perp;
    if (fabsf(diff) < tol) {
      found = 1;
    } else if (diff > 0.0f) {
      min_beta = beta;
      beta = (max_beta == FLT_MAX || max_beta == -FLT_MAX) ? beta * 2.0f : (beta + max_beta) * 0.5f;
    } else {
      max_beta = beta;
      beta = (min_beta == -FLT_MAX || min_beta == FLT_MAX) ? beta * 0.5f : (beta + min_beta) * 0.5f;
    }
  }
  const float inv_sum_p = 1.0f / sum_p;
  for (int j = 0; j < k; ++j) p[j] *= inv_sum_p;
}

typedef struct {
  uint64_t key;
  float value;
} packed_edge;

static int packed_edge_cmp(const void* a, const void* b) {
  const uint64_t ka = ((const packed_edge*)a)->key;
  const uint64_t kb = ((const packed_edge*)b)->key;
  return ka < kb ? -1 : (ka > kb ? 1 : 0);
}

long long or_tsne_build_p(const int* idx_cm, const float* dist_cm, int n, int k, int index_offset,
                          double perplexity, int* row_ptr, int* col, float* val) {
  if (n < 2 || k < 1) return -1;
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < k; ++j) {
      const int nb = idx_cm[(size_t)j * n + i] - index_offset;
      const float d = dist_cm[(size_t)j * n + i];
      if (nb < 0 || nb >= n) return -1;
      if (!isfinite(d) || d < 0.0f) return -1;
    }
  }
  packed_edge* edges = (packed_edge*)malloc(sizeof(packed_edge) * (size_t)n * k);
  float* row_d = (float*)malloc(sizeof(float) * (size_t)k);
  float* row_p = (float*)malloc(sizeof(float) * (size_t)k);
  size_t m = 0;
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < k; ++j) row_d[j] = dist_cm[(size_t)j * n + i];
    or_tsne_row_probabilities(row_d, k, perplexity, row_p);
    for (int j = 0; j < k; ++j) {
      const int nb = idx_cm[(size_t)j * n + i] - index_offset;
      if (nb == i) continue;
      const uint32_t a = (uint32_t)(i < nb ? i : nb);
      const uint32_t b = (uint32_t)(i < nb ? nb : i);
      edges[m].key = ((uint64_t)a << 32) | b;
      edges[m].value = row_p[j];
      ++m;
    }
  }
  free(row_d);
  free(row_p);
  qsort(edges, m, sizeof(packed_edge), packed_edge_cmp);

  for (int i = 0; i <= n; ++i) row_ptr[i] = 0;
  size_t write = 0;
  double total = 0.0;
  for (size_t read = 0; read < m;) {
    const uint64_t key = edges[read].key;
    double sum = 0.0;
    while (read < m && edges[read].key == key) {
      sum += (double)edges[read].value;
      ++read;
    }
    edges[write].key = key;
    edges[write].value = (float)sum;
    ++write;
    total += sum;
    ++row_ptr[(key >> 32) + 1];
    ++row_ptr[(key & 0xffffffffu) + 1];
  }
  if (write == 0 || !isfinite(total) || total <= 0.0) {
    free(edges);
    return -1;
  }
  for (int i = 0; i < n; ++i) row_ptr[i + 1] += row_ptr[i];
  int* fill = (int*)malloc(sizeof(int) * (size_t)n);
  for (int i = 0; i < n; ++i) fill[i] = row_ptr[i];
  const float norm = (float)(0.5 / total);
  for (size_t e = 0; e < write; ++e) {
    const int a = (int)(edges[e].key >> 32);
    const int b = (int)(edges[e].key & 0xffffffffu);
    const float value = edges[e].value * norm;
    int pos = fill[a]++;
    col[pos] = b;
    val[pos] = value;
    pos = fill[b]++;
    col[pos] = a;
    val[pos] = value;
  }
  free(fill);
  free(edges);
  return (long long)row_ptr[n];
}

/* ------------------------------------------------------------------ */
/* t-SNE: gradient                                                     */
/* ------------------------------------------------------------------ */

/* In-place iterative radix-2 complex FFT in double (size a power of two). */
static void fft_double(double* re, double* im, int m, int inverse) {
  for (int i = 1, j = 0; i < m; ++i) {
    int bit = m >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) {
      double t = re[i]; re[i] = re[j]; re[j] = t;
      t = im[i]; im[i] = im[j]; im[j] = t;
    }
  }
  const double sign = inverse ? 1.0 : -1.0;
  for (int len = 2; len <= m; len <<= 1) {
    const int half = len >> 1;
    for (int j = 0; j < half; ++j) {
      const double ang = sign * 2.0 * M_PI * (double)j / (double)len;
      const double wr = cos(ang);
      const double wi = sin(ang);
      for (int i = 0; i < m; i += len) {
        const int u = i + j;
        const int v = u + half;
        const double xr = re[v] * wr - im[v] * wi;
        const double xi = re[v] * wi + im[v] * wr;
        re[v] = re[u] - xr;
        im[v] = im[u] - xi;
        re[u] += xr;
        im[u] += xi;
      }
    }
  }
}

/* 2-D transform of an m x m plane (row-major). */
static void fft2_double(double* re, double* im, int m, int inverse) {
  double* cr = (double*)malloc(sizeof(double) * (size_t)m);
  double* ci = (double*)malloc(sizeof(double) * (size_t)m);
  for (int r = 0; r < m; ++r) fft_double(re + (size_t)r * m, im + (size_t)r * m, m, inverse);
  for (int c = 0; c < m; ++c) {
    for (int r = 0; r < m; ++r) { cr[r] = re[(size_t)r * m + c]; ci[r] = im[(size_t)r * m + c]; }
    fft_double(cr, ci, m, inverse);
    for (int r = 0; r < m; ++r) { re[(size_t)r * m + c] = cr[r]; im[(size_t)r * m + c] = ci[r]; }
  }
  free(cr);
  free(ci);
}

/* bilinear_grid_value_t<float>, src/tsne_neighbors.cpp:760-781. */
static float bilinear_value(const float* grid, int g, float gx, float gy) {
  const float cx = fmaxf(0.0f, fminf((float)(g - 1), gx));
  const float cy = fmaxf(0.0f, fminf((float)(g - 1), gy));
  int x0 = (int)floorf(cx);
  int y0 = (int)floorf(cy);
  if (x0 > g - 2) x0 = g - 2;
  if (x0 < 0) x0 = 0;
  if (y0 > g - 2) y0 = g - 2;
  if (y0 < 0) y0 = 0;
  const float tx = cx - (float)x0;
  const float ty = cy - (float)y0;
  const float v00 = grid[(size_t)y0 * g + x0];
  const float v10 = grid[(size_t)y0 * g + x0 + 1];
  const float v01 = grid[(size_t)(y0 + 1) * g + x0];
  const float v11 = grid[(size_t)(y0 + 1) * g + x0 + 1];
  return (1.0f - tx) * (1.0f - ty) * v00 + tx * (1.0f - ty) * v10 + (1.0f - tx) * ty * v01 +
         tx * ty * v11;
}

void or_tsne_repulsive_fft(const float* y, int n, int grid_size, float* grad, double* out_z) {
  const int g = grid_size;
  const int m = g << 1;
  const size_t gt = (size_t)g * g;
  const size_t mt = (size_t)m * m;

  /* Layout bounds and grid geometry, :1090-1106. */
  float min_x = y[0], max_x = y[0], min_y = y[1], max_y = y[1];
  for (int i = 1; i < n; ++i) {
    min_x = fminf(min_x, y[2 * i]);
    max_x = fmaxf(max_x, y[2 * i]);
    min_y = fminf(min_y, y[2 * i + 1]);
    max_y = fmaxf(max_y, y[2 * i + 1]);
  }
  const float cx = 0.5f * (min_x + max_x);
  const float cy = 0.5f * (min_y + max_y);
  float span = fmaxf(max_x - min_x, max_y - min_y);
  if (!isfinite(span) || span <= 0.0f) span = 1.0f;
  const float half = 0.55f * span + 1.0e-3f;
  const float lower_x = cx - half;
  const float lower_y = cy - half;
  const float spacing = (2.0f * half) / (float)(g - 1);
  const float inv_spacing = 1.0f / spacing;

  /* Bilinear charge splat, :1112-1148 (serial, point order). */
  float* mass = (float*)calloc(gt, sizeof(float));
  float* mass_x = (float*)calloc(gt, sizeof(float));
  float* mass_y = (float*)calloc(gt, sizeof(float));
  float* gxs = (float*)malloc(sizeof(float) * (size_t)n);
  float* gys = (float*)malloc(sizeof(float) * (size_t)n);
  for (int i = 0; i < n; ++i) {
    const float xc = y[2 * i];
    const float yc = y[2 * i + 1];
    const float raw_x = (xc - lower_x) * inv_spacing;
    const float raw_y = (yc - lower_y) * inv_spacing;
    const float clx = fmaxf(0.0f, fminf((float)(g - 1), raw_x));
    const float cly = fmaxf(0.0f, fminf((float)(g - 1), raw_y));
    int x0 = (int)floorf(clx);
    int y0 = (int)floorf(cly);
    if (x0 > g - 2) x0 = g - 2;
    if (x0 < 0) x0 = 0;
    if (y0 > g - 2) y0 = g - 2;
    if (y0 < 0) y0 = 0;
    const float tx = clx - (float)x0;
    const float ty = cly - (float)y0;
    gxs[i] = clx;
    gys[i] = cly;
    const float w00 = (1.0f - tx) * (1.0f - ty);
    const float w10 = tx * (1.0f - ty);
    const float w01 = (1.0f - tx) * ty;
    const float w11 = tx * ty;
    const size_t p00 = (size_t)y0 * g + x0;
    const size_t p10 = p00 + 1;
    const size_t p01 = p00 + g;
    const size_t p11 = p01 + 1;
    mass[p00] += w00; mass[p10] += w10; mass[p01] += w01; mass[p11] += w11;
    mass_x[p00] += w00 * xc; mass_x[p10] += w10 * xc; mass_x[p01] += w01 * xc; mass_x[p11] += w11 * xc;
    mass_y[p00] += w00 * yc; mass_y[p10] += w10 * yc; mass_y[p01] += w01 * yc; mass_y[p11] += w11 * yc;
  }

  /* Linear convolution on the zero-padded 2g x 2g torus, :880-942.  Kernel
   * samples are formed in float exactly as the reference forms them. */
  double* kq_re = (double*)calloc(mt, sizeof(double));
  double* kq_im = (double*)calloc(mt, sizeof(double));
  double* kq2_re = (double*)calloc(mt, sizeof(double));
  double* kq2_im = (double*)calloc(mt, sizeof(double));
  for (int dy = -(g - 1); dy <= g - 1; ++dy) {
    const int yy = dy < 0 ? dy + m : dy;
    const float y_off = (float)dy * spacing;
    for (int dx = -(g - 1); dx <= g - 1; ++dx) {
      const int xx = dx < 0 ? dx + m : dx;
      const float x_off = (float)dx * spacing;
      const float d2 = x_off * x_off + y_off * y_off;
      const float q = 1.0f / (1.0f + d2);
      const float q2 = q * q;
      kq_re[(size_t)yy * m + xx] = (double)q;
      kq2_re[(size_t)yy * m + xx] = (double)q2;
    }
  }
  fft2_double(kq_re, kq_im, m, 0);
  fft2_double(kq2_re, kq2_im, m, 0);

  const float* charges[3] = {mass, mass_x, mass_y};
  double* spec_re[3];
  double* spec_im[3];
  for (int c = 0; c < 3; ++c) {
    spec_re[c] = (double*)calloc(mt, sizeof(double));
    spec_im[c] = (double*)calloc(mt, sizeof(double));
    for (int r = 0; r < g; ++r)
      for (int x = 0; x < g; ++x) spec_re[c][(size_t)r * m + x] = (double)charges[c][(size_t)r * g + x];
    fft2_double(spec_re[c], spec_im[c], m, 0);
  }
  /* phi_q = m*Kq, phi_q2 = m*Kq2, phi_xq2 = mx*Kq2, phi_yq2 = my*Kq2. */
  const int src_charge[4] = {0, 0, 1, 2};
  const int use_q2[4] = {0, 1, 1, 1};
  float* pot[4];
  double* wr = (double*)malloc(sizeof(double) * mt);
  double* wi = (double*)malloc(sizeof(double) * mt);
  for (int o = 0; o < 4; ++o) {
    const double* ar = spec_re[src_charge[o]];
    const double* ai = spec_im[src_charge[o]];
    const double* br = use_q2[o] ? kq2_re : kq_re;
    const double* bi = use_q2[o] ? kq2_im : kq_im;
    for (size_t t = 0; t < mt; ++t) {
      wr[t] = ar[t] * br[t] - ai[t] * bi[t];
      wi[t] = ar[t] * bi[t] + ai[t] * br[t];
    }
    fft2_double(wr, wi, m, 1);
    pot[o] = (float*)malloc(sizeof(float) * gt);
    const double scale = 1.0 / (double)mt;
    for (int r = 0; r < g; ++r)
      for (int x = 0; x < g; ++x) pot[o][(size_t)r * g + x] = (float)(wr[(size_t)r * m + x] * scale);
  }

  /* Normalisation Z and the repulsive gather, :1150-1180. */
  double sum_q = 0.0;
  for (int i = 0; i < n; ++i) sum_q += (double)bilinear_value(pot[0], g, gxs[i], gys[i]);
  double z = sum_q - (double)n;
  if (out_z != NULL) *out_z = z;
  const float inv_sum_q = (float)(1.0 / fmax(z, (double)FLT_MIN));
  for (int i = 0; i < n; ++i) {
    const float q2v = bilinear_value(pot[1], g, gxs[i], gys[i]);
    const float xq2v = bilinear_value(pot[2], g, gxs[i], gys[i]);
    const float yq2v = bilinear_value(pot[3], g, gxs[i], gys[i]);
    grad[2 * i] = -(y[2 * i] * q2v - xq2v) * inv_sum_q;
    grad[2 * i + 1] = -(y[2 * i + 1] * q2v - yq2v) * inv_sum_q;
  }

  for (int o = 0; o < 4; ++o) free(pot[o]);
  for (int c = 0; c < 3; ++c) { free(spec_re[c]); free(spec_im[c]); }
  free(wr); free(wi);
  free(kq_re); free(kq_im); free(kq2_re); free(kq2_im);
  free(mass); free(mass_x); free(mass_y); free(gxs); free(gys);
}

void or_tsne_attractive(const int* row_ptr, const int* col, const float* val, int n,
                        const float* y, float exaggeration, float* grad) {
  for (int i = 0; i < n; ++i) {
    for (int pos = row_ptr[i]; pos < row_ptr[i + 1]; ++pos) {
      const int j = col[pos];
      const float d0 = y[2 * i] - y[2 * j];
      const float d1 = y[2 * i + 1] - y[2 * j + 1];
      float d2 = 0.0f;
      d2 += d0 * d0;
      d2 += d1 * d1;
      const float q = 1.0f / (1.0f + d2);
      const float coeff = exaggeration * val[pos] * q;
      grad[2 * i] += coeff * d0;
      grad[2 * i + 1] += coeff * d1;
    }
  }
}

void or_tsne_gradient_fft(const int* row_ptr, const int* col, const float* val, int n,
                          const float* y, float exaggeration, int grid_size, float* grad,
                          double* out_z) {
  or_tsne_repulsive_fft(y, n, grid_size, grad, out_z);
  or_tsne_attractive(row_ptr, col, val, n, y, exaggeration, grad);
}

void or_tsne_gradient_exact(const int* row_ptr, const int* col, const float* val, int n,
                            const float* y, float exaggeration, float* grad) {
  float* g = (float*)calloc((size_t)n * 2, sizeof(float));
  double sum_q = 0.0;
  for (int i = 0; i < n - 1; ++i) {
    for (int j = i + 1; j < n; ++j) {
      const float e0 = y[2 * i] - y[2 * j];
      const float e1 = y[2 * i + 1] - y[2 * j + 1];
      float d2 = 0.0f;
      d2 += e0 * e0;
      d2 += e1 * e1;
      const float q = 1.0f / (1.0f + d2);
      sum_q += 2.0 * (double)q;
      const float coeff = -(q * q);
      const float s0 = coeff * e0;
      const float s1 = coeff * e1;
      g[2 * i] += s0; g[2 * j] -= s0;
      g[2 * i + 1] += s1; g[2 * j + 1] -= s1;
    }
  }
  const float inv = (float)(1.0 / fmax(sum_q, (double)FLT_MIN));
  for (int t = 0; t < 2 * n; ++t) grad[t] = g[t] * inv;
  free(g);
  or_tsne_attractive(row_ptr, col, val, n, y, exaggeration, grad);
}

static float sign_f(float x) { return x == 0.0f ? 0.0f : (x < 0.0f ? -1.0f : 1.0f); }

void or_tsne_update(float* y, float* update, float* gains, const float* grad, int n,
                    float learning_rate, float momentum, float min_gain, float max_step_norm) {
  const int clip = isfinite(max_step_norm) && max_step_norm > 0.0f;
  const float max_sq = max_step_norm * max_step_norm;
  for (int i = 0; i < n; ++i) {
    float norm_sq = 0.0f;
    for (int d = 0; d < 2; ++d) {
      const int t = 2 * i + d;
      if (sign_f(update[t]) != sign_f(grad[t])) gains[t] += 0.2f;
      else gains[t] = gains[t] * 0.8f + min_gain;
      if (gains[t] < min_gain) gains[t] = min_gain;
      update[t] = momentum * update[t] - learning_rate * gains[t] * grad[t];
      norm_sq += update[t] * update[t];
    }
    float scale = 1.0f;
    if (clip && norm_sq > max_sq) scale = max_step_norm / sqrtf(fmaxf(norm_sq, FLT_MIN));
    for (int d = 0; d < 2; ++d) {
      const int t = 2 * i + d;
      update[t] *= scale;
      y[t] += update[t];
    }
  }
  or_tsne_zero_mean(y, n);
}

void or_tsne_zero_mean(float* y, int n) {
  double mx = 0.0, my = 0.0;
  for (int i = 0; i < n; ++i) { mx += y[2 * i]; my += y[2 * i + 1]; }
  mx /= (double)n;
  my /= (double)n;
  const float fx = (float)mx, fy = (float)my;
  for (int i = 0; i < n; ++i) { y[2 * i] -= fx; y[2 * i + 1] -= fy; }
}

double or_tsne_kl(const int* row_ptr, const int* col, const float* val, int n, const float* y) {
  double sum_q = 0.0;
  for (int i = 0; i < n - 1; ++i) {
    for (int j = i + 1; j < n; ++j) {
      const float e0 = y[2 * i] - y[2 * j];
      const float e1 = y[2 * i + 1] - y[2 * j + 1];
      float d2 = 0.0f;
      d2 += e0 * e0;
      d2 += e1 * e1;
      sum_q += 2.0 / (1.0 + (double)d2);
    }
  }
  const double zq = (double)(float)fmax(sum_q, (double)FLT_MIN);
  double total = 0.0;
  for (int i = 0; i < n; ++i) {
    double row = 0.0;
    for (int pos = row_ptr[i]; pos < row_ptr[i + 1]; ++pos) {
      const int j = col[pos];
      const float e0 = y[2 * i] - y[2 * j];
      const float e1 = y[2 * i + 1] - y[2 * j + 1];
      float d2 = 0.0f;
      d2 += e0 * e0;
      d2 += e1 * e1;
      const double p = (double)val[pos];
      const double q = (1.0 / (1.0 + (double)d2)) / zq;
      row += p * log((p + 1e-9) / (q + 1e-9));
    }
    total += row;
  }
  return total;
}

int or_tsne_run(const int* row_ptr, const int* col, const float* val, int n, const float* init,
                int early_exaggeration_iter, int n_iter, float early_exaggeration,
                float exaggeration, float learning_rate, int learning_rate_auto,
                float initial_momentum, float final_momentum, float min_gain,
                float max_step_norm, int grid_size, float* out) {
  const size_t m = (size_t)n * 2;
  float* y = out;
  memcpy(y, init, sizeof(float) * m);
  or_tsne_zero_mean(y, n);
  float* grad = (float*)calloc(m, sizeof(float));
  float* upd = (float*)calloc(m, sizeof(float));
  float* gains = (float*)malloc(sizeof(float) * m);
  for (size_t t = 0; t < m; ++t) gains[t] = 1.0f;
  for (int phase = 0; phase < 2; ++phase) {
    const int iters = phase == 0 ? early_exaggeration_iter : n_iter;
    const float ex = phase == 0 ? early_exaggeration : exaggeration;
    const float mom = phase == 0 ? initial_momentum : final_momentum;
    const float lr = learning_rate_auto ? (float)((double)n / fmax((double)ex, DBL_MIN)) : learning_rate;
    for (int it = 0; it < iters; ++it) {
      or_tsne_gradient_fft(row_ptr, col, val, n, y, ex, grid_size, grad, NULL);
      or_tsne_update(y, upd, gains, grad, n, lr, mom, min_gain, max_step_norm);
    }
  }
  free(grad);
  free(upd);
  free(gains);
  return 0;
}

void or_tsne_iterate(const int* row_ptr, const int* col, const float* val, int n, float* y,
                     float* update, float* gains, int iters, float exaggeration, float momentum,
                     float learning_rate, float min_gain, float max_step_norm, int grid_size) {
  float* grad = (float*)calloc((size_t)n * 2, sizeof(float));
  for (int it = 0; it < iters; ++it) {
    or_tsne_gradient_fft(row_ptr, col, val, n, y, exaggeration, grid_size, grad, NULL);
    or_tsne_update(y, update, gains, grad, n, learning_rate, momentum, min_gain, max_step_norm);
  }
  free(grad);
}

/* ------------------------------------------------------------------ */
/* UMAP                                                                */
/* ------------------------------------------------------------------ */

float or_umap_powf(float x, float b) {
  if (x <= 0.0f) return 0.0f;
  uint32_t bits;
  memcpy(&bits, &x, sizeof(bits));
  const float bias_word = 1064866805.0f;
  const int whole = (int)b;
  const float frac = b - (float)whole;
  const uint32_t interp = (uint32_t)(frac * ((float)bits - bias_word) + bias_word);
  float frac_pow;
  memcpy(&frac_pow, &interp, sizeof(frac_pow));
  float int_pow = 1.0f;
  float base = x;
  int e = whole;
  while (e > 0) {
    if (e & 1) int_pow *= base;
    base *= base;
    e >>= 1;
  }
  return int_pow * frac_pow;
}

int or_umap_positive_samples(float period, int epoch) {
  if (period <= 0.0f || !isfinite(period) || epoch == 0) return 0;
  const float now = (float)epoch;
  const float prev = (float)(epoch - 1);
  const int cur = (int)floorf(now / period);
  const int old = (int)floorf(prev / period);
  const int s = cur - old;
  return s > 0 ? s : 0;
}

int or_umap_negative_samples(float period, int negative_sample_rate, int epoch) {
  if (negative_sample_rate <= 0 || period <= 0.0f || !isfinite(period) || epoch == 0) return 0;
  const float now = (float)epoch;
  const float prev = (float)(epoch - 1);
  const int cur = (int)floorf(now / period);
  const int old = (int)floorf(prev / period);
  if (cur <= old) return 0;
  const float neg_period = period / (float)negative_sample_rate;
  if (neg_period <= 0.0f || !isfinite(neg_period)) return 0;
  const int cur_total = (int)floorf((now - neg_period) / neg_period);
  int prev_total = 0;
  if (cur > 1) {
    const float prev_active = ceilf((float)(cur - 1) * period);
    prev_total = (int)floorf((prev_active - neg_period) / neg_period);
  }
  const int s = cur_total - prev_total;
  return s > 0 ? s : 0;
}

static uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

int or_umap_negative_vertex(int n, uint32_t seed, int epoch, int head, uint32_t key, int sample) {
  uint32_t x = seed;
  x ^= (uint32_t)epoch * 0x9e3779b9u;
  x ^= ((uint32_t)head + 1u) * 0x85ebca6bu;
  x ^= (key + 1u) * 0xc2b2ae35u;
  x ^= ((uint32_t)sample + 1u) * 0x27d4eb2du;
  return (int)(mix32(x) % (uint32_t)n);
}

void or_umap_find_ab(double spread, double min_dist, double* a_out, double* b_out) {
  if (fabs(spread - 1.0) < 1e-12 && fabs(min_dist - 0.01) < 1e-12) {
    *a_out = 1.895605865596314; *b_out = 0.8006377738365004; return;
  }
  if (fabs(spread - 1.0) < 1e-12 && fabs(min_dist - 0.1) < 1e-12) {
    *a_out = 1.5769434601962196; *b_out = 0.8950608781227859; return;
  }
  if (fabs(spread - 1.0) < 1e-12 && fabs(min_dist - 0.5) < 1e-12) {
    *a_out = 0.5830300199018228; *b_out = 1.3341669931033755; return;
  }
  double xs[300], ys[300];
  for (int i = 0; i < 300; ++i) {
    xs[i] = (spread * 3.0) * (double)i / 299.0;
    ys[i] = xs[i] < min_dist ? 1.0 : exp(-(xs[i] - min_dist) / spread);
  }
  double best_a = 1.5769434601962196, best_b = 0.8950608781227859, best_loss = INFINITY;
  for (double loga = -4.0; loga <= 4.0001; loga += 0.2) {
    for (double b = 0.25; b <= 2.0001; b += 0.05) {
      const double a = exp(loga);
      double loss = 0.0;
      for (int i = 0; i < 300; ++i) {
        const double yhat = 1.0 / (1.0 + a * pow(xs[i], 2.0 * b));
        const double e = yhat - ys[i];
        loss += e * e;
      }
      if (loss < best_loss) { best_loss = loss; best_a = a; best_b = b; }
    }
  }
  for (int iter = 0; iter < 80; ++iter) {
    double ga = 0.0, gb = 0.0;
    for (int i = 0; i < 300; ++i) {
      const double x = fmax(xs[i], 1e-6);
      const double x2b = pow(x, 2.0 * best_b);
      const double den = 1.0 + best_a * x2b;
      const double e = 1.0 / den - ys[i];
      ga += e * (-x2b / (den * den));
      gb += e * (-(best_a * x2b * 2.0 * log(x)) / (den * den));
    }
    best_a = fmax(1e-4, best_a - 0.01 * ga);
    best_b = fmax(0.1, best_b - 0.01 * gb);
  }
  *a_out = best_a;
  *b_out = best_b;
}

static float clip4(float v) { return v < -4.0f ? -4.0f : (v > 4.0f ? 4.0f : v); }

/* Attractive coefficient (objective 0), src/fast_knn_umap.cpp:4985-4987. */
static float attr_coeff(float d2, float a, float b) {
  const float d2b = or_umap_powf(d2, b);
  return -2.0f * a * b * (d2b / d2) / (a * d2b + 1.0f);
}

/* Repulsive coefficient (objective 0), src/fast_knn_umap.cpp:5013-5014. */
static float rep_coeff(float d2, float a, float b, float gamma) {
  const float d2b = or_umap_powf(d2, b);
  return gamma * 2.0f * b / ((0.001f + d2) * (a * d2b + 1.0f));
}

void or_umap_epoch_delta(const int* heads, const int* tails, const float* eps_per_sample,
                         int n_edges, float* layout, int n, int epoch, int n_epochs,
                         int negative_sample_rate, float learning_rate, float a, float b,
                         float gamma, uint32_t seed, int hash_key_is_tail, float max_abs_coord) {
  const float eps = 1.1920928955078125e-7f;
  double* delta = (double*)calloc((size_t)n * 2, sizeof(double));
  const float alpha = learning_rate * (1.0f - (float)epoch / fmaxf(1.0f, (float)n_epochs));
  for (int e = 0; e < n_edges; ++e) {
    const int h = heads[e];
    const int t = tails[e];
    if (h < 0 || h >= n || t < 0 || t >= n || h == t) continue;
    const float per = eps_per_sample[e];
    const int pos = or_umap_positive_samples(per, epoch);
    if (pos <= 0) continue;
    for (int s = 0; s < pos; ++s) {
      const float dx = layout[2 * h] - layout[2 * t];
      const float dy = layout[2 * h + 1] - layout[2 * t + 1];
      const float d2 = fmaxf(eps, dx * dx + dy * dy);
      const float c = attr_coeff(d2, a, b);
      const float gx = clip4(c * dx) * alpha;
      const float gy = clip4(c * dy) * alpha;
      delta[2 * h] += gx; delta[2 * h + 1] += gy;
      delta[2 * t] -= gx; delta[2 * t + 1] -= gy;
    }
    const int ns = or_umap_negative_samples(per, negative_sample_rate, epoch);
    for (int s = 0; s < ns; ++s) {
      const uint32_t key = hash_key_is_tail ? (uint32_t)t : (uint32_t)e;
      const int k = or_umap_negative_vertex(n, seed, epoch, h, key, s);
      if (k == h || k == t) continue;
      const float dx = layout[2 * h] - layout[2 * k];
      const float dy = layout[2 * h + 1] - layout[2 * k + 1];
      const float d2 = fmaxf(eps, dx * dx + dy * dy);
      const float c = rep_coeff(d2, a, b, gamma);
      delta[2 * h] += clip4(c * dx) * alpha;
      delta[2 * h + 1] += clip4(c * dy) * alpha;
    }
  }
  for (int i = 0; i < n; ++i) {
    for (int d = 0; d < 2; ++d) {
      float v = layout[2 * i + d] + (float)delta[2 * i + d];
      if (!isfinite(v)) v = 0.0f;
      v = fminf(max_abs_coord, fmaxf(-max_abs_coord, v));
      layout[2 * i + d] = v;
    }
  }
  free(delta);
}

void or_umap_replay_serial(const int* heads, const int* tails, const float* eps_per_sample,
                           int n_edges, float* layout, int n, int epoch_begin, int epoch_end,
                           int n_epochs, int negative_sample_rate, float learning_rate, float a,
                           float b, float gamma, uint32_t seed, int hash_key_is_tail,
                           int sanitize_each_epoch) {
  const float eps = 1.1920928955078125e-7f;
  for (int epoch = epoch_begin; epoch < epoch_end; ++epoch) {
    const float alpha = learning_rate * (1.0f - (float)epoch / fmaxf(1.0f, (float)n_epochs));
    for (int e = 0; e < n_edges; ++e) {
      const int h = heads[e];
      const int t = tails[e];
      if (h < 0 || h >= n || t < 0 || t >= n || h == t) continue;
      const float per = eps_per_sample[e];
      const int pos = or_umap_positive_samples(per, epoch);
      if (pos <= 0) continue;
      for (int s = 0; s < pos; ++s) {
        const float dx = layout[2 * h] - layout[2 * t];
        const float dy = layout[2 * h + 1] - layout[2 * t + 1];
        const float d2 = fmaxf(eps, dx * dx + dy * dy);
        const float c = attr_coeff(d2, a, b);
        const float gx = clip4(c * dx) * alpha;
        const float gy = clip4(c * dy) * alpha;
        layout[2 * h] += gx; layout[2 * h + 1] += gy;
        layout[2 * t] += -gx; layout[2 * t + 1] += -gy;
      }
      const int ns = or_umap_negative_samples(per, negative_sample_rate, epoch);
      for (int s = 0; s < ns; ++s) {
        const uint32_t key = hash_key_is_tail ? (uint32_t)t : (uint32_t)e;
        const int k = or_umap_negative_vertex(n, seed, epoch, h, key, s);
        if (k == h || k == t) continue;
        const float dx = layout[2 * h] - layout[2 * k];
        const float dy = layout[2 * h + 1] - layout[2 * k + 1];
        const float d2 = fmaxf(eps, dx * dx + dy * dy);
        const float c = rep_coeff(d2, a, b, gamma);
        layout[2 * h] += clip4(c * dx) * alpha;
        layout[2 * h + 1] += clip4(c * dy) * alpha;
      }
    }
    if (sanitize_each_epoch) {
      for (int i = 0; i < 2 * n; ++i) {
        float v = layout[i];
        if (!isfinite(v)) v = 0.0f;
        layout[i] = fminf(16.0f, fmaxf(-16.0f, v));
      }
    }
  }
}

/* smooth_knn_dist for one row, src/fast_knn_umap.cpp:925-981. */
static void smooth_row(const float* d, int k, double target, double global_mean, float* rho_out,
                       float* sigma_out) {
  const double tol = 1.0e-5;
  double rho = INFINITY, row_sum = 0.0;
  int row_count = 0;
  for (int j = 0; j < k; ++j) {
    if (!isfinite(d[j])) continue;
    if (d[j] >= 0.0f) { row_sum += (double)d[j]; ++row_count; }
    if (d[j] > 0.0f && (double)d[j] < rho) rho = (double)d[j];
  }
  if (!isfinite(rho)) rho = 0.0;
  *rho_out = (float)rho;
  const double sigma_max = DBL_MAX;
  double sigma = 1.0, best = 1.0, best_diff = sigma_max, lo = 0.0, hi = sigma_max;
  for (int iter = 0; iter < 64; ++iter) {
    double psum = 0.0;
    const double safe = fmax(sigma, 1.0e-12);
    for (int j = 0; j < k; ++j) {
      if (!isfinite(d[j])) continue;
      const double dd = (double)d[j] - rho;
      psum += dd <= 0.0 ? 1.0 : exp(-dd / safe);
    }
    const double diff = fabs(psum - target);
    if (diff < best_diff) { best_diff = diff; best = sigma; }
    if (psum > target) {
      hi = sigma;
      sigma = 0.5 * (lo + hi);
    } else {
      lo = sigma;
      if (hi == sigma_max) sigma *= 2.0;
      else sigma = 0.5 * (lo + hi);
    }
    if (diff < tol) break;
  }
  const double row_mean = row_count > 0 ? row_sum / (double)row_count : global_mean;
  const double floor_v = 1.0e-3 * (rho > 0.0 ? row_mean : global_mean);
  best = fmax(best, floor_v);
  *sigma_out = (float)fmax(best, 1.0e-12);
}

typedef struct {
  int nb;
  float w;
} nbw;

long long or_umap_graph(const int* idx_cm, const float* dist_cm, int n, int k, int index_offset,
                        int* offsets, int* neighbors, float* weights, float* eps_per_sample,
                        float* max_weight_out) {
  if (n < 2 || k < 1) return -1;
  /* Global mean of finite non-negative distances (long double), :883-914. */
  long double gsum = 0.0L;
  size_t gcount = 0;
  for (size_t t = 0; t < (size_t)n * k; ++t) {
    const float d = dist_cm[t];
    if (isfinite(d) && d >= 0.0f) { gsum += (long double)d; ++gcount; }
  }
  const double global_mean = gcount > 0 ? (double)(gsum / (long double)gcount) : 1.0;
  const double target = log2((double)k);

  /* Directed rows: weights, stable sort by neighbour, duplicates -> max, :1585-1640 and 1275-1345. */
  int* d_off = (int*)calloc((size_t)n + 1, sizeof(int));
  nbw* dir = (nbw*)malloc(sizeof(nbw) * (size_t)n * k);
  float* row_d = (float*)malloc(sizeof(float) * (size_t)k);
  nbw* row = (nbw*)malloc(sizeof(nbw) * (size_t)k);
  size_t wpos = 0;
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < k; ++j) row_d[j] = dist_cm[(size_t)j * n + i];
    float rho, sigma;
    smooth_row(row_d, k, target, global_mean, &rho, &sigma);
    int cnt = 0;
    for (int j = 0; j < k; ++j) {
      const int nb = idx_cm[(size_t)j * n + i] - index_offset;
      const float d = row_d[j];
      if (nb < 0 || nb >= n || nb == i || !isfinite(d)) continue;
      const float w = d <= rho ? 1.0f : expf(-(d - rho) / sigma);
      if (!isfinite(w) || w <= 0.0f) continue;
      /* insertion keeps equal neighbours in arrival order (stable) */
      int c = cnt;
      while (c > 0 && row[c - 1].nb > nb) { row[c] = row[c - 1]; --c; }
      row[c].nb = nb;
      row[c].w = w;
      ++cnt;
    }
    int r = 0;
    while (r < cnt) {
      const int nb = row[r].nb;
      float w = row[r].w;
      ++r;
      while (r < cnt && row[r].nb == nb) { w = fmaxf(w, row[r].w); ++r; }
      dir[wpos].nb = nb;
      dir[wpos].w = w;
      ++wpos;
    }
    d_off[i + 1] = (int)wpos;
  }
  free(row_d);
  free(row);

  /* Incoming (transposed) rows in ascending source order, :1646-1690. */
  int* in_off = (int*)calloc((size_t)n + 1, sizeof(int));
  for (size_t t = 0; t < wpos; ++t) ++in_off[dir[t].nb + 1];
  for (int i = 0; i < n; ++i) in_off[i + 1] += in_off[i];
  int* cursor = (int*)malloc(sizeof(int) * (size_t)n);
  for (int i = 0; i < n; ++i) cursor[i] = in_off[i];
  nbw* inc = (nbw*)malloc(sizeof(nbw) * (wpos > 0 ? wpos : 1));
  for (int i = 0; i < n; ++i) {
    for (int p = d_off[i]; p < d_off[i + 1]; ++p) {
      const int tgt = dir[p].nb;
      inc[cursor[tgt]].nb = i;
      inc[cursor[tgt]].w = dir[p].w;
      ++cursor[tgt];
    }
  }
  free(cursor);

  /* Fuzzy union merge f + r - f*r, drop <= 1e-6, :1692-1740. */
  offsets[0] = 0;
  size_t out = 0;
  for (int i = 0; i < n; ++i) {
    int op = d_off[i], oe = d_off[i + 1], ip = in_off[i], ie = in_off[i + 1];
    while (op < oe || ip < ie) {
      const int onb = op < oe ? dir[op].nb : INT_MAX;
      const int inb = ip < ie ? inc[ip].nb : INT_MAX;
      int nb;
      float f = 0.0f, r = 0.0f;
      if (onb == inb) { nb = onb; f = dir[op].w; r = inc[ip].w; ++op; ++ip; }
      else if (onb < inb) { nb = onb; f = dir[op].w; ++op; }
      else { nb = inb; r = inc[ip].w; ++ip; }
      if (nb == i) continue;
      const float w = f + r - f * r;
      if (!isfinite(w) || w <= 1.0e-6f) continue;
      neighbors[out] = nb;
      weights[out] = w;
      ++out;
    }
    offsets[i + 1] = (int)out;
  }
  free(d_off);
  free(dir);
  free(in_off);
  free(inc);

  /* attach_csr_epoch_schedule, :1255-1273. */
  float maxw = 0.0f;
  for (size_t t = 0; t < out; ++t)
    if (isfinite(weights[t]) && weights[t] > maxw) maxw = weights[t];
  for (size_t t = 0; t < out; ++t) {
    if (maxw <= 0.0f) eps_per_sample[t] = INFINITY;
    else eps_per_sample[t] = maxw / fmaxf(weights[t], 1.0e-6f);
  }
  *max_weight_out = maxw;
  return (long long)out;
}

/* ---------------- UMAP: device-KNN path ---------------- */

int or_umap_graph_width(int k) { return 2 * k < 256 ? 2 * k : 256; }

int or_umap_device_graph(const int* idx_cm, const float* dist_cm, int n, int k, int index_offset,
                         int binary, int* nbr, float* w) {
  const int width = or_umap_graph_width(k);
  const size_t nk = (size_t)n * k;
  int* nbr_k = (int*)malloc(nk * sizeof(int));
  float* w_k = (float*)malloc(nk * sizeof(float));
  int* slot_k = (int*)malloc(nk * sizeof(int));
  int* own = (int*)calloc((size_t)n, sizeof(int));
  if (!nbr_k || !w_k || !slot_k || !own) {
    free(nbr_k); free(w_k); free(slot_k); free(own);
    return -1;
  }
  /* prepare_directed_knn_kernel, src/embedding_cuda_kernels.cpp:1004-1058. */
  for (int i = 0; i < n; ++i) {
    float rho = INFINITY;
    for (int j = 0; j < k; ++j) {
      const float d = dist_cm[(size_t)j * n + i];
      if (d > 0.0f && d < rho) rho = d;
    }
    if (!isfinite(rho)) rho = 0.0f;
    const float target = log2f((float)(k < 2 ? 2 : k));
    float lo = 0.0f, hi = INFINITY, sigma = 1.0f;
    for (int step = 0; step < 48; ++step) {
      float psum = 0.0f;
      for (int j = 0; j < k; ++j) {
        const float d = dist_cm[(size_t)j * n + i] - rho;
        psum += d <= 0.0f ? 1.0f : expf(-d / sigma);
      }
      if (fabsf(psum - target) < 1.0e-5f) break;
      if (psum > target) {
        hi = sigma;
        sigma = 0.5f * (lo + hi);
      } else {
        lo = sigma;
        sigma = isinf(hi) ? sigma * 2.0f : 0.5f * (lo + hi);
      }
    }
    sigma = fmaxf(sigma, 1.0e-6f);
    for (int j = 0; j < k; ++j) {
      const int nb = idx_cm[(size_t)j * n + i] - index_offset;
      const float d = dist_cm[(size_t)j * n + i];
      const int valid = nb >= 0 && nb < n && nb != i;
      const float wt = valid ? (d <= rho ? 1.0f : expf(-(d - rho) / sigma)) : 0.0f;
      const size_t e = (size_t)i * k + j;
      nbr_k[e] = valid ? nb : -1;
      w_k[e] = wt;
      slot_k[e] = (valid && !(wt <= 0.0f)) ? own[i]++ : -1;
    }
  }
  for (size_t s = 0; s < (size_t)n * width; ++s) {
    nbr[s] = (int)(s / width);
    w[s] = 0.0f;
  }
  /* Own entries: add_umap_outgoing_kernel (:1111-1135); the reverse weight is
   * that of the first entry of the target row naming this row (:1060-1071). */
  for (int i = 0; i < n; ++i) {
    for (int t = 0; t < k; ++t) {
      const size_t e = (size_t)i * k + t;
      if (slot_k[e] < 0) continue;
      const int j = nbr_k[e];
      float r = 0.0f;
      for (int u = 0; u < k; ++u) {
        if (nbr_k[(size_t)j * k + u] == i) {
          r = w_k[(size_t)j * k + u];
          break;
        }
      }
      const float f = w_k[e];
      nbr[(size_t)i * width + slot_k[e]] = j;
      w[(size_t)i * width + slot_k[e]] = f + r - f * r;
    }
  }
  /* Incoming-only entries: add_umap_incoming_kernel (:1137-1160), appended in
   * ascending (source row, rank) order while the row has room. */
  int* fill = (int*)malloc((size_t)n * sizeof(int));
  for (int i = 0; i < n; ++i) fill[i] = own[i];
  for (int j = 0; j < n; ++j) {
    for (int t = 0; t < k; ++t) {
      const size_t e = (size_t)j * k + t;
      const int i = nbr_k[e];
      if (i < 0 || w_k[e] <= 0.0f) continue;
      int named = 0;
      for (int u = 0; u < k && !named; ++u) named = nbr_k[(size_t)i * k + u] == j;
      if (named) continue;
      if (fill[i] < width) {
        nbr[(size_t)i * width + fill[i]] = j;
        w[(size_t)i * width + fill[i]] = w_k[e];
      }
      ++fill[i];
    }
  }
  if (binary) {
    /* binary_graph_weights_kernel, :1099-1109. */
    for (size_t s = 0; s < (size_t)n * width; ++s) {
      const int row = (int)(s / width);
      w[s] = (nbr[s] >= 0 && nbr[s] < n && nbr[s] != row) ? 1.0f : 0.0f;
    }
  }
  free(fill);
  free(nbr_k);
  free(w_k);
  free(slot_k);
  free(own);
  return width;
}

long long or_umap_pack_coo(const int* nbr, const float* w, int n, int width, int rank_major, int* heads,
                           int* tails, float* weights, float* epochs_per_sample) {
  long long out = 0;
  const long long slots = (long long)n * width;
  for (long long id = 0; id < slots; ++id) {
    int row, slot;
    if (rank_major) {
      slot = (int)(id / n);
      row = (int)(id - (long long)slot * n);
    } else {
      row = (int)(id / width);
      slot = (int)(id - (long long)row * width);
    }
    const size_t dense = (size_t)row * width + slot;
    const int nb = nbr[dense];
    const float wt = w[dense];
    if (!(nb >= 0 && nb < n && nb != row && wt > 0.0f)) continue;
    heads[out] = row;
    tails[out] = nb;
    weights[out] = wt;
    epochs_per_sample[out] = 1.0f / fmaxf(wt, 1.0e-6f);
    ++out;
  }
  return out;
}

/* deterministic_unit, src/embedding_cuda_kernels.cpp:266-274. */
static float hashed_unit(uint32_t seed, int row, int col) {
  uint32_t x = seed;
  x ^= ((uint32_t)row + 1u) * 0x9e3779b9u;
  x ^= ((uint32_t)col + 1u) * 0x85ebca6bu;
  return (float)(mix32(x) & 0x00ffffffu) / 8388607.5f - 1.0f;
}

/* reduce/finalize_init_stats_kernel, :1198-1306. */
static void whiten_stats(const float* y, int n, double st[5]) {
  double sx = 0.0, sy = 0.0, sxx = 0.0, sxy = 0.0, syy = 0.0;
  for (int i = 0; i < n; ++i) {
    const double x = y[2 * i], v = y[2 * i + 1];
    sx += x;
    sy += v;
    sxx += x * x;
    sxy += x * v;
    syy += v * v;
  }
  const double dn = (double)(n > 1 ? n : 1);
  const double x_ss = fmax(sxx - sx * sx / dn, 1.0e-24);
  const double y_ss = fmax(syy - sy * sy / dn, 1.0e-24);
  const double xy = sxy - sx * sy / dn;
  const double norm_x = sqrt(x_ss);
  const double proj = xy / norm_x;
  const double resid = fmax(y_ss - proj * proj, 1.0e-24);
  st[0] = sx / dn;
  st[1] = sy / dn;
  st[2] = 1.0 / norm_x;
  st[3] = proj;
  st[4] = 1.0 / sqrt(resid);
}

/* normalize_init_kernel, :1308-1319. */
static void whiten_value(const float* v, const double st[5], float* out) {
  const double x = ((double)v[0] - st[0]) * st[2];
  const double yc = (double)v[1] - st[1];
  const double y = (yc - st[3] * x) * st[4];
  out[0] = (float)x;
  out[1] = (float)y;
}

void or_umap_diffusion_init(const int* nbr, const float* w, int n, int width, uint32_t seed, int iters,
                            float* out) {
  float* cur = (float*)malloc((size_t)n * 2 * sizeof(float));
  float* next = (float*)malloc((size_t)n * 2 * sizeof(float));
  for (int i = 0; i < n; ++i) {
    cur[2 * i] = hashed_unit(seed, i, 0);
    cur[2 * i + 1] = hashed_unit(seed, i, 1);
  }
  /* random_init_kernel (:1162-1167), whitened. */
  double st[5];
  whiten_stats(cur, n, st);
  for (int i = 0; i < n; ++i) whiten_value(cur + 2 * i, st, cur + 2 * i);
  /* diffuse_init_kernel, :1169-1196, each round followed by whitening. */
  for (int it = 0; it < iters; ++it) {
    for (int i = 0; i < n; ++i) {
      float sx = 0.0f, sy = 0.0f, sw = 0.0f;
      for (int j = 0; j < width; ++j) {
        const int nb = nbr[(size_t)i * width + j];
        const float wt = w[(size_t)i * width + j];
        if (nb < 0 || nb >= n || nb == i || wt <= 0.0f) continue;
        sx += wt * cur[2 * nb];
        sy += wt * cur[2 * nb + 1];
        sw += wt;
      }
      if (sw <= 0.0f) {
        next[2 * i] = cur[2 * i];
        next[2 * i + 1] = cur[2 * i + 1];
      } else {
        next[2 * i] = sx / sw;
        next[2 * i + 1] = sy / sw;
      }
    }
    whiten_stats(next, n, st);
    for (int i = 0; i < n; ++i) whiten_value(next + 2 * i, st, next + 2 * i);
    float* t = cur;
    cur = next;
    next = t;
  }
  memcpy(out, cur, (size_t)n * 2 * sizeof(float));
  free(cur);
  free(next);
}
