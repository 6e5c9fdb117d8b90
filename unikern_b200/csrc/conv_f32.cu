// conv_f32.cu -- 2-D convolution (stride 1) as an implicit GEMM on the FFMA
// pipes, with the per-output-channel scale fused into the epilogue.
// Replaces uk_conv<OCB>/uk_conv_g<OCB> and their launch plan
// (src/codegen_hip.cpp:337-411, :420-599); semantics of src/reference.cpp:6-22.
//
// GEMM view (both layouts): rows = output channels (A = the weights, K-
// contiguous), columns = output pixels over (image, ho, wo), inner dimension
// k over the filter taps.  The pixel operand is gathered from the input on
// the fly (no im2col buffer); padding reads as zero.  A CTA computes a
// BM x BN tile of (channel, pixel) with TM x TN micro-tiles per thread and a
// register-prefetched, double-buffered K loop (one barrier per slab).
//   NCHW:  k = (c, kh, kw); x index ((n*C + c)*H + hi)*W + wi
//   KML :  k = (kh, kw, c); x index ((ho+kh)*W + (wo+kw))*C + c   (N = 1, valid)
// Output pixel p = n*Ho*Wo + q is stored at (n*Oc + oc)*Ho*Wo + q, which is
// NCHW for the batch form and [Oc][Ho][Wo] for the KML form.
#include <cstdio>
#include <cstdlib>

#include "uk_common.cuh"
#include "uk_plan.cuh"

namespace {

struct ConvArgs {
  const float* x;
  const float* w;
  const float* scale;
  float* y;
  int N, C, H, W, Oc, Kh, Kw, pad, Ho, Wo;
  int64_t npix;  // N * Ho * Wo
  int K;         // C * Kh * Kw
};

template <int BM, int BN, int BK, int TM, int TN, int LAYOUT, int KS>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) k_conv(const ConvArgs a) {
  constexpr int NTX = BN / TN, NTY = BM / TM, NT = NTX * NTY;
  constexpr int A_VECS = BM * BK / 4, A_PER = (A_VECS + NT - 1) / NT;
  constexpr int B_KPT = BK * BN / NT;  // k values per thread in the B slab
  static_assert(NT % BN == 0 && (BK * BN) % NT == 0, "B slab mapping");
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % NTX, ty = tid / NTX;
  const int m0 = blockIdx.y * BM;
  const int64_t p0 = (int64_t)blockIdx.x * BN;
  const int K = a.K, M = a.Oc;
  const int Kh = KS ? KS : a.Kh, Kw = KS ? KS : a.Kw;
  const bool avec = (K % 4) == 0;

  // this thread's gather column (fixed for the whole K loop)
  const int bp = tid % BN, bk0 = (tid / BN) * B_KPT;
  const int64_t gp = p0 + bp;
  const bool pvalid = gp < a.npix;
  int n = 0, ho = 0, wo = 0;
  if (pvalid) {
    const int64_t hw = (int64_t)a.Ho * a.Wo;
    n = (int)(gp / hw);
    const int q = (int)(gp - (int64_t)n * hw);
    ho = q / a.Wo;
    wo = q - ho * a.Wo;
  }
  const float* xb;
  if (LAYOUT == UK_CONV_NCHW)
    xb = a.x + (size_t)n * a.C * a.H * a.W;
  else
    xb = a.x + ((size_t)ho * a.W + wo) * a.C;

  float ra[A_PER][4], rb[B_KPT];
  auto load_slab = [&](int k0) {
#pragma unroll
    for (int p = 0; p < A_PER; ++p) {
      const int i = tid + p * NT;
      if (i < A_VECS) {
        const int m = i / (BK / 4), kq = (i % (BK / 4)) * 4;
        const int gm = m0 + m, gk = k0 + kq;
        const float* src = a.w + (size_t)gm * K + gk;
        if (avec) {
          if (gm < M && gk < K) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(src));
            ra[p][0] = t.x; ra[p][1] = t.y; ra[p][2] = t.z; ra[p][3] = t.w;
          } else {
            ra[p][0] = ra[p][1] = ra[p][2] = ra[p][3] = 0.f;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) ra[p][j] = (gm < M && gk + j < K) ? __ldg(src + j) : 0.f;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < B_KPT; ++j) {
      const int gk = k0 + bk0 + j;
      float v = 0.f;
      if (pvalid && gk < K) {
        if (LAYOUT == UK_CONV_NCHW) {
          const int c = gk / (Kh * Kw);
          const int r = gk - c * (Kh * Kw);
          const int kh = r / Kw, kw = r - (r / Kw) * Kw;
          const int hi = ho + kh - a.pad, wi = wo + kw - a.pad;
          if (hi >= 0 && hi < a.H && wi >= 0 && wi < a.W) v = __ldg(xb + ((size_t)c * a.H + hi) * a.W + wi);
        } else {
          const int t = gk / a.C;
          const int c = gk - t * a.C;
          const int kh = t / Kw, kw = t - kh * Kw;
          v = __ldg(xb + ((size_t)kh * a.W + kw) * a.C + c);
        }
      }
      rb[j] = v;
    }
  };
  auto store_slab = [&](int buf) {
#pragma unroll
    for (int p = 0; p < A_PER; ++p) {
      const int i = tid + p * NT;
      if (i < A_VECS) {
        const int m = i / (BK / 4), kq = (i % (BK / 4)) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) As[buf][kq + j][m] = ra[p][j];
      }
    }
#pragma unroll
    for (int j = 0; j < B_KPT; ++j) Bs[buf][bk0 + j][bp] = rb[j];
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const int nslab = (K + BK - 1) / BK;
  load_slab(0);
  store_slab(0);
  __syncthreads();
  for (int s = 0; s < nslab; ++s) {
    const int buf = s & 1;
    if (s + 1 < nslab) load_slab((s + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float av[TM], bv[TN];
#pragma unroll
      for (int g = 0; g < TM / 4; ++g) {
        const float4 t = *reinterpret_cast<const float4*>(&As[buf][k][g * NTY * 4 + ty * 4]);
        av[g * 4 + 0] = t.x; av[g * 4 + 1] = t.y; av[g * 4 + 2] = t.z; av[g * 4 + 3] = t.w;
      }
#pragma unroll
      for (int g = 0; g < TN / 4; ++g) {
        const float4 t = *reinterpret_cast<const float4*>(&Bs[buf][k][g * NTX * 4 + tx * 4]);
        bv[g * 4 + 0] = t.x; bv[g * 4 + 1] = t.y; bv[g * 4 + 2] = t.z; bv[g * 4 + 3] = t.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (s + 1 < nslab) store_slab(buf ^ 1);
    __syncthreads();
  }

  // epilogue: fused per-channel scale, pixel-contiguous stores
  const int64_t hw = (int64_t)a.Ho * a.Wo;
#pragma unroll
  for (int gj = 0; gj < TN / 4; ++gj)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t p = p0 + gj * NTX * 4 + tx * 4 + j;
      if (p >= a.npix) continue;
      const int64_t pn = p / hw, q = p - pn * hw;
#pragma unroll
      for (int gi = 0; gi < TM / 4; ++gi)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int oc = m0 + gi * NTY * 4 + ty * 4 + i;
          if (oc >= M) continue;
          float v = acc[gi * 4 + i][gj * 4 + j];
          if (a.scale) v = v * __ldg(a.scale + oc);
          a.y[((size_t)pn * M + oc) * hw + q] = v;
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN, int LAYOUT>
void launch(const ConvArgs& a, cudaStream_t st) {
  constexpr int NT = (BM / TM) * (BN / TN);
  dim3 grid((unsigned)((a.npix + BN - 1) / BN), (unsigned)((a.Oc + BM - 1) / BM));
  if (a.Kh == 3 && a.Kw == 3)
    k_conv<BM, BN, BK, TM, TN, LAYOUT, 3><<<grid, NT, 0, st>>>(a);
  else if (a.Kh == 1 && a.Kw == 1)
    k_conv<BM, BN, BK, TM, TN, LAYOUT, 1><<<grid, NT, 0, st>>>(a);
  else
    k_conv<BM, BN, BK, TM, TN, LAYOUT, 0><<<grid, NT, 0, st>>>(a);
}

// UK_FFMA_CONV_PLAN="bm,bn,bk" pins one compiled tile of this kernel (a
// measurement knob, like the reference's UK_CONV_TILE for its own tiles):
// 128,128,8 / 128,128,16 / 64,64,8 / 32,64,16.  Returns false when unset;
// *bad when the value names no compiled tile.
bool pinned_conv_tile(uk::Tile* t, bool* bad) {
  *bad = false;
  const char* e = getenv("UK_FFMA_CONV_PLAN");
  if (e == nullptr || e[0] == 0) return false;
  int bm = 0, bn = 0, bk = 0;
  if (sscanf(e, "%d,%d,%d", &bm, &bn, &bk) != 3 ||
      !((bm == 128 && bn == 128 && (bk == 8 || bk == 16)) || (bm == 64 && bn == 64 && bk == 8) ||
        (bm == 32 && bn == 64 && bk == 16))) {
    *bad = true;
    return false;
  }
  *t = uk::Tile{bm, bn, bk, 2};
  return true;
}

template <int LAYOUT>
void dispatch(const ConvArgs& a, cudaStream_t st, const uk::Tile& t) {
  if (t.bm == 128 && t.bk == 16)
    launch<128, 128, 16, 8, 8, LAYOUT>(a, st);
  else if (t.bm == 128)
    launch<128, 128, 8, 8, 8, LAYOUT>(a, st);
  else if (t.bm == 64)
    launch<64, 64, 8, 4, 4, LAYOUT>(a, st);
  else
    launch<32, 64, 16, 4, 4, LAYOUT>(a, st);
}

}  // namespace

namespace uk {
int conv2d_ffma(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh, int Kw, int Oc,
                int pad, const float* scale, int layout, cudaStream_t st);
}

extern "C" int uk_cuda_conv2d_f32(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh,
                                  int Kw, int Oc, int pad, const float* scale, int layout, void* stream) {
  return uk::conv2d_ffma(X, Wt, Y, N, H, W, C, Kh, Kw, Oc, pad, scale, layout, (cudaStream_t)stream);
}

// the FFMA implicit GEMM (also the path of uk_cuda_conv2d_f32_ws for shapes
// the tensor-core kernel does not take)
int uk::conv2d_ffma(const float* X, const float* Wt, float* Y, int N, int H, int W, int C, int Kh, int Kw, int Oc,
                    int pad, const float* scale, int layout, cudaStream_t st) {
  if (layout != UK_CONV_KML && layout != UK_CONV_NCHW)
    return uk::fail(UK_EINVAL, "conv2d: unknown layout %d", layout);
  if (N < 0 || H <= 0 || W <= 0 || C <= 0 || Kh <= 0 || Kw <= 0 || Oc <= 0 || pad < 0)
    return uk::fail(UK_EINVAL, "conv2d: invalid dims N=%d H=%d W=%d C=%d Kh=%d Kw=%d Oc=%d pad=%d", N, H, W, C, Kh,
                    Kw, Oc, pad);
  if (layout == UK_CONV_KML && (N != 1 || pad != 0))
    return uk::fail(UK_EINVAL, "conv2d: the KML layout is one image with valid padding (N=1, pad=0)");
  ConvArgs a{};
  a.x = X; a.w = Wt; a.scale = scale; a.y = Y;
  a.N = N; a.C = C; a.H = H; a.W = W; a.Oc = Oc; a.Kh = Kh; a.Kw = Kw; a.pad = pad;
  a.Ho = H + 2 * pad - Kh + 1;
  a.Wo = W + 2 * pad - Kw + 1;
  if (a.Ho <= 0 || a.Wo <= 0) return uk::fail(UK_EINVAL, "conv2d: the filter is larger than the padded input");
  if ((int64_t)C * Kh * Kw > 2147483647LL) return uk::fail(UK_EINVAL, "conv2d: C*Kh*Kw too large");
  a.K = C * Kh * Kw;
  a.npix = (int64_t)N * a.Ho * a.Wo;
  if (N == 0) return UK_OK;
  if ((a.npix + 31) / 32 > 2147483647LL || (Oc + 31) / 32 > 65535) return uk::fail(UK_EINVAL, "conv2d: grid too large");
  if (int rc = uk::check_device_ptr(X, "X")) return rc;
  if (int rc = uk::check_device_ptr(Wt, "Wt")) return rc;
  if (int rc = uk::check_device_ptr(Y, "Y")) return rc;
  if (scale)
    if (int rc = uk::check_device_ptr(scale, "scale")) return rc;
  // the weight loader uses 16-byte loads when K % 4 == 0: refuse a misaligned
  // base instead of faulting
  if (!uk::aligned16(Wt) && a.K % 4 == 0) return uk::fail(UK_EINVAL, "conv2d: Wt must be 16-byte aligned");
  uk::Tile t = uk::conv_tile(a.npix, a.Oc, uk::sm_count());
  bool bad = false;
  pinned_conv_tile(&t, &bad);
  if (bad)
    return uk::fail(UK_EINVAL, "conv2d: UK_FFMA_CONV_PLAN=%s names no compiled tile (128,128,8 128,128,16 64,64,8 "
                    "32,64,16)", getenv("UK_FFMA_CONV_PLAN"));
  if (layout == UK_CONV_NCHW) dispatch<UK_CONV_NCHW>(a, st, t);
  else dispatch<UK_CONV_KML>(a, st, t);
  return uk::check_launch("conv2d");
}
