// Plain complex diagonal scan and the MIMO scan + block-diagonal readout, for sm_100a.
//
// Reference behaviour (paths relative to the reference project):
//   models/selective_lru/selective_lru_mimo_triton.py:105-211  selective scan operator
//   models/selective_lru/selective_lru_mimo_triton.py:370-462  fused MIMO scan + readout
//   models/selective_lru/selective_lru.py:550-574, 590-599    the PyTorch equivalents
//
// Complex scan: one thread per (sequence, mode) chain, flat index s * N + n so a warp
// reads 32 consecutive modes of one step; 8-step load batches issued one batch ahead.
// The backward reads the forward's saved trajectory (it is an output of the operator),
// so it needs no recompute.
//
// MIMO: one CTA per (sequence, head). Time is processed in kTC-step chunks: the mode
// threads run the recurrence for the chunk and leave h_t in shared memory, then all
// threads evaluate the chunk's readout y[t, f] = sum_n Re(C[f, n] h_t[n]) + D x. The
// backward mirrors it per chunk (last first): all threads form the readout adjoint
// g[t, n] = sum_f dy[t, f] conj(C[f, n]) into shared memory, the mode threads run
// G_t = g_t + dh_t + conj(lam_{t+1}) G_{t+1}, and all threads accumulate dC and dD for
// the chunk in shared memory. Per-(sequence, head) dC / dD rows are reduced over
// sequences by the two-stage fixed-order column sum.
#include "semx_common.cuh"
#include "semx_reduce.cuh"

namespace {

constexpr int kBlock = 128;
constexpr int kSub = 8;
constexpr int kTC = 32;  // MIMO time chunk

// ------------------------------------------------------------------- complex scan
struct CSParams {
  int64_t S, L, N;
  const float* lr;
  const float* li;
  const float* br;
  const float* bi;
  float* hr;
  float* hi;
  const float* ghr;
  const float* ghi;
  float* dlr;
  float* dli;
  float* dbr;
  float* dbi;
};

__global__ void __launch_bounds__(kBlock) cscan_fwd_kernel(const CSParams p) {
  const int64_t gid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  if (gid >= p.S * p.N) return;
  const int64_t s = gid / p.N;
  const int64_t n = gid - s * p.N;
  const int64_t base = s * p.L * p.N + n;
  const int L = (int)p.L;
  float hr = 0.f, hi = 0.f;
  for (int t0 = 0; t0 < L; t0 += kSub) {
    float a[kSub], b[kSub], u[kSub], v[kSub];
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (t0 + i < L) {
        const int64_t off = base + (int64_t)(t0 + i) * p.N;
        a[i] = __ldg(p.lr + off);
        b[i] = __ldg(p.li + off);
        u[i] = __ldg(p.br + off);
        v[i] = __ldg(p.bi + off);
      }
    }
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (t0 + i < L) {
        const float nr = a[i] * hr - b[i] * hi + u[i];
        const float ni = b[i] * hr + a[i] * hi + v[i];
        hr = nr;
        hi = ni;
        const int64_t off = base + (int64_t)(t0 + i) * p.N;
        p.hr[off] = hr;
        p.hi[off] = hi;
      }
    }
  }
}

__global__ void __launch_bounds__(kBlock) cscan_bwd_kernel(const CSParams p) {
  const int64_t gid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  if (gid >= p.S * p.N) return;
  const int64_t s = gid / p.N;
  const int64_t n = gid - s * p.N;
  const int64_t base = s * p.L * p.N + n;
  const int L = (int)p.L;
  float Gr = 0.f, Gi = 0.f;    // G_{t+1}
  float lnr = 0.f, lni = 0.f;  // lam_{t+1}
  for (int tb = L - 1; tb >= 0; tb -= kSub) {
    float gr[kSub], gi[kSub], hpr[kSub], hpi[kSub], lr[kSub], li[kSub];
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      const int t = tb - i;
      if (t >= 0) {
        const int64_t off = base + (int64_t)t * p.N;
        gr[i] = __ldg(p.ghr + off);
        gi[i] = __ldg(p.ghi + off);
        lr[i] = __ldg(p.lr + off);
        li[i] = __ldg(p.li + off);
        hpr[i] = t > 0 ? __ldg(p.hr + off - p.N) : 0.f;
        hpi[i] = t > 0 ? __ldg(p.hi + off - p.N) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      const int t = tb - i;
      if (t >= 0) {
        const float nr = gr[i] + lnr * Gr + lni * Gi;
        const float ni = gi[i] + lnr * Gi - lni * Gr;
        Gr = nr;
        Gi = ni;
        const int64_t off = base + (int64_t)t * p.N;
        p.dbr[off] = Gr;
        p.dbi[off] = Gi;
        p.dlr[off] = Gr * hpr[i] + Gi * hpi[i];
        p.dli[off] = Gi * hpr[i] - Gr * hpi[i];
        lnr = lr[i];
        lni = li[i];
      }
    }
  }
}

// --------------------------------------------------------------------------- MIMO
struct MParams {
  int64_t S, L, H, Nh, Fh;
  const float* lr;
  const float* li;
  const float* br;
  const float* bi;
  const float* Cr;
  const float* Ci;
  const float* x;
  const float* D;
  float* y;
  float* hr;
  float* hi;
  const float* dy;
  const float* dhr;
  const float* dhi;
  float* dlr;
  float* dli;
  float* dbr;
  float* dbi;
  float* dx;
  float* part;  // (S, H * (2 * Fh * Nh + Fh))
};

// Shared memory: C_re, C_im [Fh][Nh]; h_re, h_im [kTC][Nh] (forward) and, in the
// backward, additionally g_re, g_im [kTC][Nh], dy [kTC][Fh], dC_re, dC_im [Fh][Nh] and
// dD [Fh].
__global__ void __launch_bounds__(kBlock) mimo_fwd_kernel(const MParams p) {
  extern __shared__ float sm[];
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, L = (int)p.L;
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  float* Cr = sm;
  float* Ci = Cr + Fh * Nh;
  float* Hr = Ci + Fh * Nh;
  float* Hi = Hr + kTC * Nh;
  for (int i = tid; i < Fh * Nh; i += kBlock) {
    Cr[i] = p.Cr[(int64_t)h * Fh * Nh + i];
    Ci[i] = p.Ci[(int64_t)h * Fh * Nh + i];
  }
  const int64_t N = p.H * p.Nh, Fd = p.H * p.Fh;
  float st_r[2] = {0.f, 0.f}, st_i[2] = {0.f, 0.f};  // modes tid and tid + kBlock
  __syncthreads();
  for (int t0 = 0; t0 < L; t0 += kTC) {
    const int tc = min(kTC, L - t0);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int n = tid + k * kBlock;
      if (n < Nh) {
        float hr = st_r[k], hi = st_i[k];
        for (int i = 0; i < tc; ++i) {
          const int64_t off = (s * p.L + t0 + i) * N + (int64_t)h * Nh + n;
          const float a = __ldg(p.lr + off), b = __ldg(p.li + off);
          const float u = __ldg(p.br + off), v = __ldg(p.bi + off);
          const float nr = a * hr - b * hi + u;
          const float ni = b * hr + a * hi + v;
          hr = nr;
          hi = ni;
          p.hr[off] = hr;
          p.hi[off] = hi;
          Hr[i * Nh + n] = hr;
          Hi[i * Nh + n] = hi;
        }
        st_r[k] = hr;
        st_i[k] = hi;
      }
    }
    __syncthreads();
    for (int it = tid; it < tc * Fh; it += kBlock) {
      const int i = it / Fh, f = it % Fh;
      float acc = 0.f;
      for (int n = 0; n < Nh; ++n) acc += Cr[f * Nh + n] * Hr[i * Nh + n] - Ci[f * Nh + n] * Hi[i * Nh + n];
      const int64_t of = (s * p.L + t0 + i) * Fd + (int64_t)h * Fh + f;
      p.y[of] = acc + p.D[h * Fh + f] * __ldg(p.x + of);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kBlock) mimo_bwd_kernel(const MParams p) {
  extern __shared__ float sm[];
  const int Nh = (int)p.Nh, Fh = (int)p.Fh, L = (int)p.L;
  const int64_t s = blockIdx.x / p.H;
  const int h = (int)(blockIdx.x % p.H);
  const int tid = threadIdx.x;
  float* Cr = sm;
  float* Ci = Cr + Fh * Nh;
  float* Hr = Ci + Fh * Nh;
  float* Hi = Hr + kTC * Nh;
  float* Gr_s = Hi + kTC * Nh;
  float* Gi_s = Gr_s + kTC * Nh;
  float* Dy = Gi_s + kTC * Nh;
  float* dCr = Dy + kTC * Fh;
  float* dCi = dCr + Fh * Nh;
  float* dDs = dCi + Fh * Nh;
  for (int i = tid; i < Fh * Nh; i += kBlock) {
    Cr[i] = p.Cr[(int64_t)h * Fh * Nh + i];
    Ci[i] = p.Ci[(int64_t)h * Fh * Nh + i];
    dCr[i] = 0.f;
    dCi[i] = 0.f;
  }
  for (int f = tid; f < Fh; f += kBlock) dDs[f] = 0.f;
  const int64_t N = p.H * p.Nh, Fd = p.H * p.Fh;
  float Gr[2] = {0.f, 0.f}, Gi[2] = {0.f, 0.f}, lnr[2] = {0.f, 0.f}, lni[2] = {0.f, 0.f};
  __syncthreads();
  const int nchunks = (L + kTC - 1) / kTC;
  for (int c = nchunks - 1; c >= 0; --c) {
    const int t0 = c * kTC;
    const int tc = min(kTC, L - t0);
    // dy and h of the chunk into shared memory; dx = dy * D; dD partial sums.
    for (int it = tid; it < tc * Fh; it += kBlock) {
      const int i = it / Fh, f = it % Fh;
      const int64_t of = (s * p.L + t0 + i) * Fd + (int64_t)h * Fh + f;
      const float d = __ldg(p.dy + of);
      Dy[i * Fh + f] = d;
      p.dx[of] = d * p.D[h * Fh + f];
    }
    for (int it = tid; it < tc * Nh; it += kBlock) {
      const int i = it / Nh, n = it % Nh;
      const int64_t off = (s * p.L + t0 + i) * N + (int64_t)h * Nh + n;
      Hr[i * Nh + n] = p.hr[off];
      Hi[i * Nh + n] = p.hi[off];
    }
    __syncthreads();
    // Readout adjoint g[t, n] = sum_f dy[t, f] conj(C[f, n]) (+ dh).
    for (int it = tid; it < tc * Nh; it += kBlock) {
      const int i = it / Nh, n = it % Nh;
      float gr = 0.f, gi = 0.f;
      for (int f = 0; f < Fh; ++f) {
        gr += Dy[i * Fh + f] * Cr[f * Nh + n];
        gi -= Dy[i * Fh + f] * Ci[f * Nh + n];
      }
      if (p.dhr) {
        const int64_t off = (s * p.L + t0 + i) * N + (int64_t)h * Nh + n;
        gr += __ldg(p.dhr + off);
        gi += __ldg(p.dhi + off);
      }
      Gr_s[i * Nh + n] = gr;
      Gi_s[i * Nh + n] = gi;
    }
    // dC[f, n] += sum_t dy[t, f] * conj-readout of h_t;  dD[f] += sum_t dy x.
    for (int it = tid; it < Fh * Nh; it += kBlock) {
      const int f = it / Nh, n = it % Nh;
      float ar = 0.f, ai = 0.f;
      for (int i = 0; i < tc; ++i) {
        ar += Dy[i * Fh + f] * Hr[i * Nh + n];
        ai -= Dy[i * Fh + f] * Hi[i * Nh + n];
      }
      dCr[it] += ar;
      dCi[it] += ai;
    }
    for (int f = tid; f < Fh; f += kBlock) {
      float acc = 0.f;
      for (int i = 0; i < tc; ++i) {
        const int64_t of = (s * p.L + t0 + i) * Fd + (int64_t)h * Fh + f;
        acc += Dy[i * Fh + f] * __ldg(p.x + of);
      }
      dDs[f] += acc;
    }
    __syncthreads();
    // Reverse recurrence over the chunk.
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int n = tid + k * kBlock;
      if (n < Nh) {
        for (int i = tc - 1; i >= 0; --i) {
          const int t = t0 + i;
          const int64_t off = (s * p.L + t) * N + (int64_t)h * Nh + n;
          const float gr = Gr_s[i * Nh + n] + lnr[k] * Gr[k] + lni[k] * Gi[k];
          const float gi = Gi_s[i * Nh + n] + lnr[k] * Gi[k] - lni[k] * Gr[k];
          Gr[k] = gr;
          Gi[k] = gi;
          p.dbr[off] = gr;
          p.dbi[off] = gi;
          float hpr = 0.f, hpi = 0.f;
          if (i > 0) {
            hpr = Hr[(i - 1) * Nh + n];
            hpi = Hi[(i - 1) * Nh + n];
          } else if (t > 0) {
            hpr = p.hr[off - N];
            hpi = p.hi[off - N];
          }
          p.dlr[off] = gr * hpr + gi * hpi;
          p.dli[off] = gi * hpr - gr * hpi;
          lnr[k] = __ldg(p.lr + off);
          lni[k] = __ldg(p.li + off);
        }
      }
    }
    __syncthreads();
  }
  // Per-(sequence, head) partial row: [dC_re (H,Fh,Nh) | dC_im (H,Fh,Nh) | dD (H*Fh)].
  const int64_t FN = p.H * p.Fh * p.Nh;
  float* row = p.part + s * (2 * FN + Fd);
  for (int i = tid; i < Fh * Nh; i += kBlock) {
    row[(int64_t)h * Fh * Nh + i] = dCr[i];
    row[FN + (int64_t)h * Fh * Nh + i] = dCi[i];
  }
  for (int f = tid; f < Fh; f += kBlock) row[2 * FN + (int64_t)h * Fh + f] = dDs[f];
}

size_t mimo_fwd_smem(const SemxMimoArgs* a) {
  return (size_t)(2 * a->Fh * a->Nh + 2 * kTC * a->Nh) * sizeof(float);
}
size_t mimo_bwd_smem(const SemxMimoArgs* a) {
  return (size_t)(4 * a->Fh * a->Nh + 4 * kTC * a->Nh + kTC * a->Fh + a->Fh) * sizeof(float);
}
int64_t mimo_row(const SemxMimoArgs* a) { return 2 * a->H * a->Fh * a->Nh + a->H * a->Fh; }

}  // namespace

extern "C" {

size_t semx_complex_scan_args_size(void) { return sizeof(SemxComplexScanArgs); }

int semx_complex_scan_fwd(const SemxComplexScanArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxComplexScanArgs);
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->N >= 0, SEMX_ERR_SHAPE, "complex_scan: negative size");
  if (a->S * a->L * a->N == 0) return SEMX_OK;
  SEMX_REQUIRE(a->lam_re && a->lam_im && a->Bu_re && a->Bu_im && a->h_re && a->h_im, SEMX_ERR_NULL,
               "complex_scan: NULL operand");
  int rc = semx::bind_device({a->h_re});
  if (rc != SEMX_OK) return rc;
  CSParams p = {a->S, a->L, a->N, a->lam_re, a->lam_im, a->Bu_re, a->Bu_im, a->h_re, a->h_im};
  cscan_fwd_kernel<<<(unsigned)semx::cdiv(a->S * a->N, kBlock), kBlock, 0, semx::as_stream(stream)>>>(p);
  return semx::check_launch("cscan_fwd_kernel");
}

int semx_complex_scan_bwd(const SemxComplexScanArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxComplexScanArgs);
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->N >= 0, SEMX_ERR_SHAPE, "complex_scan: negative size");
  if (a->S * a->L * a->N == 0) return SEMX_OK;
  SEMX_REQUIRE(a->lam_re && a->lam_im && a->h_re && a->h_im && a->dh_re && a->dh_im && a->dlam_re &&
                   a->dlam_im && a->dBu_re && a->dBu_im,
               SEMX_ERR_NULL, "complex_scan bwd: NULL operand");
  int rc = semx::bind_device({a->dBu_re});
  if (rc != SEMX_OK) return rc;
  CSParams p = {a->S,   a->L,     a->N,     a->lam_re,  a->lam_im,  a->Bu_re,  a->Bu_im,
                a->h_re, a->h_im, a->dh_re, a->dh_im,  a->dlam_re, a->dlam_im, a->dBu_re,
                a->dBu_im};
  cscan_bwd_kernel<<<(unsigned)semx::cdiv(a->S * a->N, kBlock), kBlock, 0, semx::as_stream(stream)>>>(p);
  return semx::check_launch("cscan_bwd_kernel");
}

size_t semx_mimo_args_size(void) { return sizeof(SemxMimoArgs); }

size_t semx_mimo_workspace_bytes(const SemxMimoArgs* a) {
  if (a == nullptr || a->S < 0 || a->H < 0 || a->Fh < 0 || a->Nh < 0) return 0;
  const int64_t K = mimo_row(a);
  return ((size_t)a->S * K + semx::colsum_group_floats(a->S, K)) * sizeof(float);
}

static int mimo_validate(const SemxMimoArgs* a) {
  SEMX_REQUIRE(a->S >= 0 && a->L >= 0 && a->H >= 0 && a->Nh >= 0 && a->Fh >= 0, SEMX_ERR_SHAPE,
               "mimo: negative size");
  SEMX_REQUIRE(a->Nh <= 2 * kBlock, SEMX_ERR_UNSUPPORTED, "mimo: Nh=%lld > %d", (long long)a->Nh,
               2 * kBlock);
  SEMX_REQUIRE(a->S * a->H <= 0x7fffffffLL, SEMX_ERR_SHAPE, "mimo: S*H too large");
  return SEMX_OK;
}

int semx_mimo_fwd(const SemxMimoArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxMimoArgs);
  int rc = mimo_validate(a);
  if (rc != SEMX_OK) return rc;
  if (a->S * a->H == 0 || a->L == 0) return SEMX_OK;
  SEMX_REQUIRE(a->lam_re && a->lam_im && a->Bu_re && a->Bu_im && a->C_re && a->C_im && a->x && a->D &&
                   a->y && a->h_re && a->h_im,
               SEMX_ERR_NULL, "mimo: NULL operand");
  rc = semx::bind_device({a->y});
  if (rc != SEMX_OK) return rc;
  MParams p = {};
  p.S = a->S; p.L = a->L; p.H = a->H; p.Nh = a->Nh; p.Fh = a->Fh;
  p.lr = a->lam_re; p.li = a->lam_im; p.br = a->Bu_re; p.bi = a->Bu_im;
  p.Cr = a->C_re; p.Ci = a->C_im; p.x = a->x; p.D = a->D; p.y = a->y; p.hr = a->h_re; p.hi = a->h_im;
  const size_t smem = mimo_fwd_smem(a);
  SEMX_REQUIRE(smem <= 227 * 1024, SEMX_ERR_UNSUPPORTED, "mimo: Fh*Nh too large for shared memory");
  if (!semx::allow_smem(mimo_fwd_kernel, smem)) return SEMX_ERR_LAUNCH;
  mimo_fwd_kernel<<<(unsigned)(a->S * a->H), kBlock, smem, semx::as_stream(stream)>>>(p);
  return semx::check_launch("mimo_fwd_kernel");
}

int semx_mimo_bwd(const SemxMimoArgs* a, semx_stream_t stream) {
  SEMX_CHECK_ARGS(a, SemxMimoArgs);
  int rc = mimo_validate(a);
  if (rc != SEMX_OK) return rc;
  cudaStream_t st = semx::as_stream(stream);
  const int64_t K = mimo_row(a);
  if (a->S * a->H == 0) return SEMX_OK;
  SEMX_REQUIRE(a->workspace != nullptr, SEMX_ERR_WORKSPACE, "mimo bwd: workspace is NULL");
  rc = semx::bind_device({a->workspace});
  if (rc != SEMX_OK) return rc;
  float* ws = reinterpret_cast<float*>(a->workspace);
  if (a->L > 0) {
    SEMX_REQUIRE(a->lam_re && a->lam_im && a->C_re && a->C_im && a->x && a->D && a->h_re && a->h_im &&
                     a->dy && a->dlam_re && a->dlam_im && a->dBu_re && a->dBu_im && a->dx,
                 SEMX_ERR_NULL, "mimo bwd: NULL operand");
    SEMX_REQUIRE((a->dh_re == nullptr) == (a->dh_im == nullptr), SEMX_ERR_NULL,
                 "mimo bwd: dh_re and dh_im must both be given or both NULL");
    MParams p = {};
    p.S = a->S; p.L = a->L; p.H = a->H; p.Nh = a->Nh; p.Fh = a->Fh;
    p.lr = a->lam_re; p.li = a->lam_im; p.Cr = a->C_re; p.Ci = a->C_im; p.x = a->x; p.D = a->D;
    p.hr = a->h_re; p.hi = a->h_im; p.dy = a->dy; p.dhr = a->dh_re; p.dhi = a->dh_im;
    p.dlr = a->dlam_re; p.dli = a->dlam_im; p.dbr = a->dBu_re; p.dbi = a->dBu_im; p.dx = a->dx;
    p.part = ws;
    const size_t smem = mimo_bwd_smem(a);
    SEMX_REQUIRE(smem <= 227 * 1024, SEMX_ERR_UNSUPPORTED, "mimo bwd: Fh*Nh too large for shared memory");
    if (!semx::allow_smem(mimo_bwd_kernel, smem)) return SEMX_ERR_LAUNCH;
    mimo_bwd_kernel<<<(unsigned)(a->S * a->H), kBlock, smem, st>>>(p);
    rc = semx::check_launch("mimo_bwd_kernel");
    if (rc != SEMX_OK) return rc;
  } else {
    cudaMemsetAsync(ws, 0, (size_t)a->S * K * sizeof(float), st);
  }
  semx::Segments seg = {};
  seg.n = 3;
  seg.out[0] = a->dC_re;
  seg.out[1] = a->dC_im;
  seg.out[2] = a->dD;
  seg.len[0] = seg.len[1] = a->H * a->Fh * a->Nh;
  seg.len[2] = a->H * a->Fh;
  return semx::colsum(ws, a->S, K, ws + (size_t)a->S * K, seg, st);
}

}  // extern "C"
