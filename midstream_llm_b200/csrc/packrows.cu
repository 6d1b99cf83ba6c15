// Packed training / validation rows gathered on the device.
//
// The reference builds each [seq+1] row on the host by copying document spans
// out of uint16 token shards and writing an end-of-document token after every
// document that ends inside the row (Midstream-LLM src/jishui/data.py:233-330
// PackedBatchIterator._fill_row, :333-379 SequentialBatchIterator._fill_row),
// then copies the int32 rows to the GPU and widens them to int64
// (pretrain_torch.py:38-40). Here the host only decides the spans (the same
// random draws, so the rows are identical); the tokens stay resident in HBM and
// one kernel writes the int64 rows.
//
// A row is a list of runs (dst column, src token, count), sorted by dst and
// covering [0, width) exactly; src < 0 means `count` copies of the token value
// -src - 1 (the end-of-document marker). One thread per output token finds its
// run by binary search; loads and stores are coalesced along the row.
#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {
namespace pack {

__global__ void pack_rows_kernel(const uint16_t* __restrict__ tokens, int64_t ntokens, const int64_t* __restrict__ runs,
                                 const int32_t* __restrict__ row_start, int width, int64_t* __restrict__ out,
                                 int* status) {
  const int row = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= width) return;
  int lo = row_start[row], hi = row_start[row + 1] - 1;  // last run with dst <= col
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (runs[3 * mid] <= col) lo = mid;
    else hi = mid - 1;
  }
  const int64_t dst = runs[3 * lo], src = runs[3 * lo + 1], count = runs[3 * lo + 2];
  int64_t v;
  if (col < dst || col >= dst + count) {
    v = -1;  // the plan does not cover this column
    atomicExch(status, 401);
  } else if (src < 0) {
    v = -src - 1;
  } else {
    const int64_t s = src + (col - dst);
    if (s < ntokens) {
      v = tokens[s];
    } else {
      v = -1;
      atomicExch(status, 402);
    }
  }
  out[(int64_t)row * width + col] = v;
}

}  // namespace pack
}  // namespace jx

using namespace jx;

extern "C" int jx_pack_rows(const void* tokens, int64_t ntokens, const int64_t* runs, const int32_t* row_start,
                            int rows, int width, int64_t* out, jx_stream_t stream) {
  JX_CHECK_ARG(tokens && runs && row_start && out, "jx_pack_rows: NULL argument");
  JX_CHECK_ARG(rows > 0 && rows <= 65535 && width > 0 && ntokens > 0, "jx_pack_rows: bad shape rows=%d width=%d",
               rows, width);
  dim3 grid((width + 255) / 256, rows);
  pack::pack_rows_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(tokens), ntokens, runs, row_start, width, out, status_ptr());
  JX_CHECK_LAUNCH("jx_pack_rows");
  return JX_OK;
}
