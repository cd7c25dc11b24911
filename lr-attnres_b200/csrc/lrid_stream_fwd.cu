// Forward instantiations of the streaming LRID read kernel (lrid_stream.cuh).
// The forward's register arrays depend on the source count only through the
// number of 32-source copy rounds, so it has two size variants, each with no
// output norm or the norm's registers for 4 or 8 chunks.
#include "lrid_stream.cuh"

namespace attnres {

template <typename T, int KP, int NORM>
static WarpFn fwd_s(int S) {
  if (S <= 32) return lrid_stream_kernel<T, KP, 32, false, NORM>;
  return lrid_stream_kernel<T, KP, 64, false, NORM>;
}

template <typename T, int KP>
static WarpFn fwd_k(int S, int nc) {
  if (nc == 0) return fwd_s<T, KP, 0>(S);
  return nc <= 4 ? fwd_s<T, KP, 4>(S) : fwd_s<T, KP, kNormMaxChunks>(S);
}

template <typename T>
static WarpFn fwd_t(int kp, int S, int nc) {
  return kp == 1 ? fwd_k<T, 1>(S, nc) : fwd_k<T, 4>(S, nc);
}

// norm_chunks: 512-byte chunks per output-norm group (0 without the norm).
WarpFn stream_kernel_fwd(int dtype, int key_packs, int S, int norm) {
  switch (dtype) {
    case ATTNRES_DTYPE_F32: return fwd_t<float>(key_packs, S, norm);
    case ATTNRES_DTYPE_F16: return fwd_t<__half>(key_packs, S, norm);
    default: return fwd_t<__nv_bfloat16>(key_packs, S, norm);
  }
}

cudaError_t stream_status_fwd(unsigned* status, bool reset) {
  return read_stream_status_word(&g_warp_status, status, reset);
}

}  // namespace attnres
