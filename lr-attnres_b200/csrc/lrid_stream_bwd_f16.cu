// Backward instantiations of the streaming LRID read kernel (lrid_stream.cuh)
// for __half: per-source gradient sums live in registers, so there is one
// variant per source-count class, with and without the output norm.
#include "lrid_stream.cuh"

namespace attnres {

template <int KP, int NORM>
static WarpFn bwd_s(int S) {
  if (S <= 16) return lrid_stream_kernel<__half, KP, 16, true, NORM>;
  if (S <= 20) return lrid_stream_kernel<__half, KP, 20, true, NORM>;
  if (S <= 24) return lrid_stream_kernel<__half, KP, 24, true, NORM>;
  if (S <= 32) return lrid_stream_kernel<__half, KP, 32, true, NORM>;
  return lrid_stream_kernel<__half, KP, 64, true, NORM>;
}

WarpFn stream_kernel_bwd_f16(int key_packs, int S, bool norm) {
  if (key_packs == 1) return norm ? bwd_s<1, 1>(S) : bwd_s<1, 0>(S);
  return norm ? bwd_s<4, 1>(S) : bwd_s<4, 0>(S);
}

cudaError_t stream_status_bwd_f16(unsigned* status, bool reset) {
  return read_stream_status_word(&g_warp_status, status, reset);
}

}  // namespace attnres
