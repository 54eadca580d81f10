// Tiled VAE decode: the latent's overlapping square tiles gathered into one
// batch (decoded together by a decoder created for the tile's size, each
// batch item normalised on its own as a tile run alone is), and the decoded
// tiles crossfaded back into the image.
//
// The reference runs the tiles one after another through one tile-sized
// graph and blends on the host (TiledVaeDecoder.Run,
// src/NaiveDiffusion/Vae/TiledVae.cs:136-159; CopyTile :67-82, BlendTile
// :84-105, DivideByWeights :107-121). The blend here is a gather: one thread
// per output cell visits the tiles that cover it in the reference's order
// (tile rows, then tile columns) and does the same float operations
// (products and sums rounded one at a time, then a correctly rounded
// reciprocal of the weight sum), so for the same tiles the image is
// bit-identical to the reference's.
#include <algorithm>
#include <climits>
#include <cstdint>
#include <string>

#include "nd_common.cuh"
#include "nd_internal.h"
#include "nd_runtime.h"

namespace nd {

namespace {

constexpr int kMaxTileStarts = 256;
constexpr int kMaxBlendChannels = 16;

struct TileGrid {
  int rows[kMaxTileStarts];
  int cols[kMaxTileStarts];
  int n_rows, n_cols;
};

__global__ void tile_gather_kernel(const float* __restrict__ latent, int channels, int height, int width,
                                   const TileGrid grid, int tile, float* __restrict__ tiles, long long total) {
  const long long plane = static_cast<long long>(height) * width;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(idx % tile);
    long long r = idx / tile;
    const int y = static_cast<int>(r % tile);
    r /= tile;
    const int c = static_cast<int>(r % channels);
    const int t = static_cast<int>(r / channels);
    const int i = t / grid.n_cols, j = t - i * grid.n_cols;
    tiles[idx] = latent[c * plane + static_cast<long long>(grid.rows[i] + y) * width + grid.cols[j] + x];
  }
}

__global__ void tile_blend_kernel(const float* __restrict__ tiles, int channels, int side, const TileGrid grid,
                                  const float* __restrict__ vertical, const float* __restrict__ horizontal,
                                  float* __restrict__ out, int height, int width) {
  const long long plane = static_cast<long long>(height) * width;
  const long long tile_plane = static_cast<long long>(side) * side;
  for (long long cell = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; cell < plane;
       cell += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int y = static_cast<int>(cell / width), x = static_cast<int>(cell - static_cast<long long>(y) * width);
    float acc[kMaxBlendChannels];
#pragma unroll
    for (int c = 0; c < kMaxBlendChannels; ++c) acc[c] = 0.f;
    float weight = 0.f;
    for (int i = 0; i < grid.n_rows; ++i) {
      const int ty = y - grid.rows[i];
      if (ty < 0 || ty >= side) continue;
      for (int j = 0; j < grid.n_cols; ++j) {
        const int tx = x - grid.cols[j];
        if (tx < 0 || tx >= side) continue;
        // VaeTiling.Window: the two axes' ramps multiplied, one float product.
        const float blend = __fmul_rn(vertical[ty], horizontal[tx]);
        const float* src = tiles + static_cast<long long>(i * grid.n_cols + j) * channels * tile_plane +
                           static_cast<long long>(ty) * side + tx;
#pragma unroll
        for (int c = 0; c < kMaxBlendChannels; ++c)
          if (c < channels) acc[c] = __fadd_rn(acc[c], __fmul_rn(src[c * tile_plane], blend));
        weight = __fadd_rn(weight, blend);
      }
    }
    const float scale = __fdiv_rn(1.0f, weight);
#pragma unroll
    for (int c = 0; c < kMaxBlendChannels; ++c)
      if (c < channels) out[c * plane + cell] = __fmul_rn(acc[c], scale);
  }
}

int fill_grid(TileGrid& g, const int32_t* rows, int n_rows, const int32_t* cols, int n_cols, int side,
              int height, int width, const char* what) {
  if (!rows || !cols || n_rows <= 0 || n_cols <= 0 || n_rows > kMaxTileStarts || n_cols > kMaxTileStarts)
    return fail(ND_ERR_INVALID, std::string(what) + ": 1 to 256 tile rows and columns");
  g.n_rows = n_rows;
  g.n_cols = n_cols;
  for (int i = 0; i < n_rows; ++i) {
    if (rows[i] < 0 || rows[i] > height - side)
      return fail(ND_ERR_INVALID, std::string(what) + ": a tile row lies outside the image");
    g.rows[i] = rows[i];
  }
  for (int j = 0; j < n_cols; ++j) {
    if (cols[j] < 0 || cols[j] > width - side)
      return fail(ND_ERR_INVALID, std::string(what) + ": a tile column lies outside the image");
    g.cols[j] = cols[j];
  }
  return ND_OK;
}

unsigned grid_for(long long work) {
  const long long cap = static_cast<long long>(sm_count()) * 16;
  return static_cast<unsigned>(std::max(1LL, std::min((work + 255) / 256, cap)));
}

}  // namespace

}  // namespace nd

int nd_op_tile_gather(const float* latent, int channels, int height, int width, const int32_t* rows, int n_rows,
                      const int32_t* cols, int n_cols, int tile, float* tiles, void* stream) {
  using namespace nd;
  if (!latent || !tiles) return fail(ND_ERR_INVALID, "tile_gather: null operand");
  if (channels <= 0 || height <= 0 || width <= 0 || tile <= 0 || tile > height || tile > width)
    return fail(ND_ERR_INVALID, "tile_gather: bad shape");
  TileGrid g;
  int rc = fill_grid(g, rows, n_rows, cols, n_cols, tile, height, width, "tile_gather");
  if (rc) return rc;
  const long long total = static_cast<long long>(n_rows) * n_cols * channels * tile * tile;
  tile_gather_kernel<<<grid_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(latent, channels, height,
                                                                                       width, g, tile, tiles, total);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}

int nd_op_tile_blend(const float* tiles, int channels, int side, const int32_t* rows, int n_rows,
                     const int32_t* cols, int n_cols, const float* vertical, const float* horizontal, float* out,
                     int height, int width, void* stream) {
  using namespace nd;
  if (!tiles || !vertical || !horizontal || !out) return fail(ND_ERR_INVALID, "tile_blend: null operand");
  if (channels <= 0 || channels > kMaxBlendChannels)
    return fail(ND_ERR_UNSUPPORTED, "tile_blend: 1 to 16 channels");
  if (height <= 0 || width <= 0 || side <= 0 || side > height || side > width)
    return fail(ND_ERR_INVALID, "tile_blend: bad shape");
  TileGrid g;
  int rc = fill_grid(g, rows, n_rows, cols, n_cols, side, height, width, "tile_blend");
  if (rc) return rc;
  tile_blend_kernel<<<grid_for(static_cast<long long>(height) * width), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(tiles, channels, side, g, vertical, horizontal, out,
                                                           height, width);
  ND_CUDA(cudaGetLastError());
  return ND_OK;
}
