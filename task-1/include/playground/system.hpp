// Types and build-time parameters of the playground task-1 harness, re-created for this repository.
// Mirrors the reference header results/naive_cycle4/include/playground/system.hpp:1-47: the element
// types (float16_t = CUDA half), and params::DataType / params::MatmulVersion selected at build time
// by TEST_FLOAT16 / TEST_FLOAT32 and MATMUL_VERSION.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <string_view>

namespace playground
{
using size_t = std::size_t;
using float64_t = double;
using float32_t = float;
using float16_t = half;
static_assert(sizeof(float16_t) == 2, "float16_t is binary16");
static_assert(sizeof(float32_t) == 4, "float32_t is binary32");
}  // namespace playground

namespace playground::params
{
#if defined(TEST_FLOAT16)
using DataType = float16_t;
constexpr std::string_view DataTypeName = "float16";
#else
using DataType = float32_t;
constexpr std::string_view DataTypeName = "float32";
#endif

#ifndef MATMUL_VERSION
#define MATMUL_VERSION 0  // v0 = cBLAS ground truth on the CPU
#endif
constexpr auto MatmulVersion = static_cast<std::uint8_t>(MATMUL_VERSION);
}  // namespace playground::params
