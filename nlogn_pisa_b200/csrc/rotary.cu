// Split-half rotary position encoding of the token mixer's queries and keys
// (pisa/pisa/ops/lrpe/rotary_torch.py:5-9, frequencies as
// xmixers/xmixers/modules/pes/lrpe.py:20-27): for i < D/2 with angle
// a = position * frequency[i] (fp32),
//   out[i]       = x[i] cos a - x[i + D/2] sin a
//   out[i + D/2] = x[i] sin a + x[i + D/2] cos a
// in fp32, rounded to the tensor's dtype.  One thread per (token, head, i),
// HBM-bound; `out` may alias `x`.
#include "internal.h"

namespace pisa {

namespace {

template <typename T>
__global__ void rotary_kernel(const T* __restrict__ x, int64_t sb, int64_t st, int64_t sh, T* out, int64_t osb,
                              int64_t ost, int64_t osh, const int64_t* __restrict__ positions, int64_t pos_sb,
                              int64_t pos_offset, const float* __restrict__ freq, int T_, int H, int half,
                              int64_t total) {
  const int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (idx >= total) return;
  const int i = int(idx % half);
  int64_t r = idx / half;
  const int h = int(r % H);
  r /= H;
  const int t = int(r % T_);
  const int b = int(r / T_);
  const int64_t pos = positions ? positions[b * pos_sb + t] : pos_offset + t;
  const float angle = float(pos) * freq[i];
  float s, c;
  sincosf(angle, &s, &c);
  const T* xp = x + b * sb + t * st + h * sh;
  const float a0 = to_f32<T>(xp[i]), a1 = to_f32<T>(xp[i + half]);
  T* op = out + b * osb + t * ost + h * osh;
  op[i] = from_f32<T>(a0 * c - a1 * s);
  op[i + half] = from_f32<T>(a0 * s + a1 * c);
}

template <typename T>
int rotary_t(const void* x, int64_t sb, int64_t st, int64_t sh, void* out, int64_t osb, int64_t ost, int64_t osh,
             const int64_t* positions, int64_t pos_sb, int64_t pos_offset, const float* freq, int64_t B,
             int64_t T_, int64_t H, int64_t D, cudaStream_t stream) {
  const int64_t total = B * T_ * H * (D / 2);
  if (total == 0) return PISA_OK;
  rotary_kernel<T><<<unsigned((total + 255) / 256), 256, 0, stream>>>(
      static_cast<const T*>(x), sb, st, sh, static_cast<T*>(out), osb, ost, osh, positions, pos_sb, pos_offset,
      freq, int(T_), int(H), int(D / 2), total);
  PISA_CHECK_LAUNCH();
  return PISA_OK;
}

}  // namespace

}  // namespace pisa

extern "C" {

int pisa_rotary(const void* x, int64_t x_sb, int64_t x_st, int64_t x_sh, void* out, int64_t out_sb, int64_t out_st,
                int64_t out_sh, const int64_t* positions, int64_t positions_sb, int64_t position_offset,
                const float* frequency, int dtype, int64_t B, int64_t T, int64_t H, int64_t D,
                pisa_stream_t stream) {
  if (dtype < PISA_F32 || dtype > PISA_F16) return pisa::fail(PISA_ERR_UNSUPPORTED, "rotary supports FP16, BF16 and FP32");
  if (B < 0 || T < 0 || H < 0 || D < 0 || D % 2) return pisa::fail(PISA_ERR_INVALID, "rotary needs an even head dimension");
  if (!x || !out || !frequency) return pisa::fail(PISA_ERR_INVALID, "x, out and frequency are required");
  if (B * T * H * (D / 2) >= (int64_t(1) << 40)) return pisa::fail(PISA_ERR_UNSUPPORTED, "tensor too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PISA_F32:
      return pisa::rotary_t<float>(x, x_sb, x_st, x_sh, out, out_sb, out_st, out_sh, positions, positions_sb,
                                   position_offset, frequency, B, T, H, D, s);
    case PISA_BF16:
      return pisa::rotary_t<__nv_bfloat16>(x, x_sb, x_st, x_sh, out, out_sb, out_st, out_sh, positions,
                                           positions_sb, position_offset, frequency, B, T, H, D, s);
    default:
      return pisa::rotary_t<__half>(x, x_sb, x_st, x_sh, out, out_sb, out_st, out_sh, positions, positions_sb,
                                    position_offset, frequency, B, T, H, D, s);
  }
}

}  // extern "C"
