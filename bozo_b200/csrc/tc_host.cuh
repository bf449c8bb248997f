// tc_host.cuh — host helpers shared by the tcgen05 kernels: TMA tensor maps
// over [B,T,H,64] bf16 views and device queries.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace bozo {

constexpr int kTcTile = 128;  // rows per TMA tile (queries or keys)
constexpr int kTcHD = 64;     // head dim of the tensor-core kernels

// True when x can be addressed by make_tmap_bthd (bf16, unit HD stride,
// 16-byte aligned base and 16-byte multiple strides on stepped dims).
bool tma_view_ok(const DevT4& x, int B, int T, int H);

// 4-D tiled tensor map over x[B,T,H,64]: dims (d, h, t, b), box
// (64, 1, box_t, 1), 128-byte swizzle, zero fill out of bounds.
bool make_tmap_bthd(CUtensorMap* m, const void* base, long long sb, long long st, long long sh,
                    int B, int T, int H, int box_t);

// 2-D tiled tensor map over a row-major bf16 (or fp32) matrix [outer, inner]
// with the given row pitch: box (box_inner, box_outer), 128-byte swizzle
// (box_inner × element size = 128 bytes), zero fill out of bounds.
bool make_tmap_2d(CUtensorMap* m, const void* base, bool f32, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

bool tmap_encoder_available();
int num_sms();

}  // namespace bozo
