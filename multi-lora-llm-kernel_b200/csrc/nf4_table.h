// NF4 (4-bit NormalFloat, QLoRA) constants shared by the NF4 kernels.
//
// kNf4Half: fp16 bit patterns of the 16 NF4 values in increasing order: the
// quantiles of N(0, 1) with delta = 1 - (1/32 + 1/30) / 2 (8 positive, 7
// negative, and 0), normalised to [-1, 1].  kNf4Mid: fp32 bit patterns of the
// 15 decision points halfway between consecutive values (computed from the
// unrounded values).  A test recomputes both from the construction.
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#define PERSONA_NF4_TABLE __device__ constexpr
#else
#define PERSONA_NF4_TABLE constexpr
#endif

namespace persona {

PERSONA_NF4_TABLE uint16_t kNf4Half[16] = {0xBC00, 0xB992, 0xB833, 0xB652, 0xB48D, 0xB1EA, 0xADD4, 0x0000,
                                   0x2D18, 0x3126, 0x33E0, 0x3568, 0x370D, 0x3880, 0x39C9, 0x3C00};
PERSONA_NF4_TABLE uint32_t kNf4Mid[15] = {0xBF591CD9, 0xBF1C5270, 0xBEEB847D, 0xBEADEA74, 0xBE703CE9,
                                  0xBE0D38B9, 0xBD3A7869, 0x3D22FB01, 0x3DF64860, 0x3E5067DC,
                                  0x3E9582D2, 0x3EC753F6, 0x3F006D02, 0x3F248DAC, 0x3F5C89D8};

// Tiled storage: one chunk per 128 x 128 tile of W[N, K].
constexpr int kNf4Tile = 128;
constexpr int kNf4Block = 64;                          // weights per absmax
constexpr int kNf4CodeBytes = kNf4Tile * kNf4Tile / 2;  // 8192
constexpr int kNf4ScaleOff = kNf4CodeBytes;             // int8 scale codes, row * 2 + half
constexpr int kNf4S127Off = kNf4ScaleOff + kNf4Tile * 2;  // fp32 s127
constexpr int kNf4ChunkBytes = kNf4S127Off + 16;        // 8464, a multiple of 16
constexpr int kNf4MaxProblems = 4;
constexpr int kNf4MaxRows = 64;                          // rows of x per GEMM launch

}  // namespace persona
