// The reference's CPU hl_quant API (encode_*, decode_*, quantize_reference,
// dequantize_reference[_to_fp16]) and the host emulation of its flat FP8 decoder, called
// exactly as the reference's own tests call them (tests/project2/test_dequant.cpp,
// test_quant_encode.cpp, test_dequant_cuda.cpp) and linked against libhlkv.so alone.
//
//   test_quant_api <dir>
//
// reads inputs that the Python side wrote to <dir> (encode_in.bin, k_scales.bin, and the
// quantize cases listed in q_cases.txt), writes every result as raw little-endian arrays
// to <dir> for comparison with the golden fixtures, and runs the known-answer and argument
// checks below.  Prints "<checks> checks, <failures> failures".
#include <algorithm>
#include <bit>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <limits>
#include <span>
#include <string>
#include <vector>

#include "hl_quant/cpu_dequant.hpp"
#include "hl_quant/cpu_quant.hpp"
#include "hl_quant/cuda_dequant.hpp"
#include "hl_quant/quant_types.hpp"

using namespace hl::quant;

namespace {

int g_checks = 0, g_failures = 0;

void check(bool ok, const std::string& what) {
  ++g_checks;
  if (!ok) {
    ++g_failures;
    std::printf("FAIL: %s\n", what.c_str());
  }
}

template <typename T>
std::vector<T> read_raw(const std::string& path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  std::vector<T> v(static_cast<std::size_t>(f.tellg()) / sizeof(T));
  f.seekg(0);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
  return v;
}

template <typename T>
void write_raw(const std::string& path, const std::vector<T>& v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
}

std::uint32_t bits(float x) { return std::bit_cast<std::uint32_t>(x); }

std::vector<std::byte> as_bytes(std::initializer_list<unsigned> v) {
  std::vector<std::byte> out;
  for (unsigned x : v) out.push_back(static_cast<std::byte>(x));
  return out;
}

// Known answers of the reference's tests (test_dequant.cpp, test_quant_encode.cpp).
void known_answers() {
  check(decode_fp8_e4m3(0x7E) == 448.0f, "E4M3 0x7E = 448");
  check(decode_fp8_e4m3(0x78) == 256.0f, "E4M3 0x78 = 256");
  check(decode_fp8_e4m3(0x01) == std::ldexp(1.0f, -9), "E4M3 0x01 = 2^-9");
  check(std::isnan(decode_fp8_e4m3(0x7F)) && std::isnan(decode_fp8_e4m3(0xFF)), "E4M3 S.1111.111 is NaN");
  check(std::isinf(decode_fp8_e5m2(0x7C)) && decode_fp8_e5m2(0xFC) < 0.0f, "E5M2 S.11111.00 is Inf");
  check(std::isnan(decode_fp8_e5m2(0x7D)), "E5M2 S.11111.01 is NaN");
  check(decode_fp8_e5m2(0x7B) == 57344.0f, "E5M2 0x7B = 57344");
  check(bits(decode_fp16(0x8000)) == 0x80000000u, "FP16 -0 decodes to -0");
  check(decode_fp16(0x0001) == std::ldexp(1.0f, -24), "FP16 smallest subnormal");
  check(bits(decode_fp16(0xFE01)) == 0xFFC00000u, "FP16 negative NaN decodes to the quiet NaN of its sign");

  check(encode_fp8_e4m3(464.0f) == 0x7E, "e4(464) = 0x7E (tie to even, below saturation)");
  check(encode_fp8_e4m3(480.0f) == 0x7E, "e4(480) saturates to 0x7E");
  check(encode_fp8_e4m3(std::numeric_limits<float>::infinity()) == 0x7E, "e4(+Inf) = 0x7E");
  check(encode_fp8_e4m3(-std::numeric_limits<float>::infinity()) == 0xFE, "e4(-Inf) = 0xFE");
  check(encode_fp8_e4m3(std::ldexp(1.0f, -10)) == 0x00, "e4(2^-10) = 0x00 (tie to even zero)");
  check(encode_fp8_e4m3(3.0f * std::ldexp(1.0f, -10)) == 0x02, "e4(3 x 2^-10) = 0x02");
  check(encode_fp8_e4m3(std::nanf("")) == 0x7F, "e4(NaN) = 0x7F");
  check(encode_fp8_e5m2(1e9f) == 0x7B, "e5(1e9) saturates to 0x7B");
  check(encode_fp8_e5m2(-std::nanf("")) == 0xFF, "e5(-NaN) = 0xFF");
  check(encode_fp16(65520.0f) == 0x7C00, "h(65520) overflows to Inf");
  check(encode_fp16(65519.0f) == 0x7BFF, "h(65519) = 65504");
  check(encode_fp16(-std::nanf("")) == 0xFE00, "h(-NaN) = 0xFE00");
  check(encode_fp16(std::ldexp(1.0f, -25)) == 0x0000, "h(2^-25) = +0 (tie to even)");
  check(encode_fp16(std::ldexp(3.0f, -26)) == 0x0001, "h(3 x 2^-26) = the smallest subnormal");

  // INT4 bytes {0x21, 0xF0, 0x0E}: low nibble first -> {1, 2, 0, 15, 14}.
  {
    const auto packed = as_bytes({0x21, 0xF0, 0x0E});
    const AffineParams p[1] = {{1.0f, 0.0f}};
    std::vector<float> out(5);
    check(dequantize_reference(QuantFormat::kInt4Packed, packed, 5, p, 6, out) == QuantStatus::kOk,
          "INT4 dequantize status");
    check(out == std::vector<float>({1, 2, 0, 15, 14}), "INT4 low nibble first");
  }
  // One rounding in the INT4 fma: q * scale + bias with scale = 1 + 2^-23, q = 15, bias = -15.
  {
    const auto packed = as_bytes({0x0F});
    const AffineParams p[1] = {{1.0f + std::ldexp(1.0f, -23), -15.0f}};
    std::vector<float> out(2);
    check(dequantize_reference(QuantFormat::kInt4Packed, packed, 2, p, 2, out) == QuantStatus::kOk, "fma status");
    check(out[0] == 15.0f * std::ldexp(1.0f, -23), "INT4 value is one fused rounding");
  }
  // INT4 padding: an odd count leaves the high nibble of the last byte zero.
  {
    const float in[3] = {0.0f, 15.0f, 7.0f};
    AffineParams p[1];
    std::byte packed[2] = {std::byte{0xAA}, std::byte{0xAA}};
    check(quantize_reference(QuantFormat::kInt4Packed, in, 4, p, packed) == QuantStatus::kOk, "INT4 odd count");
    check(packed[0] == std::byte{0xF0} && packed[1] == std::byte{0x07}, "INT4 padding nibble is zero");
    check(p[0].scale == 1.0f && p[0].bias == 0.0f, "INT4 params {1, 0}");
  }
  // FP8 scale 3/448 for amax 3.
  {
    const float in[4] = {1.0f, -3.0f, 2.0f, 0.5f};
    AffineParams p[1];
    std::byte packed[4];
    check(quantize_reference(QuantFormat::kFp8E4M3, in, 4, p, packed) == QuantStatus::kOk, "FP8 quantize");
    check(p[0].scale == 3.0f / 448.0f && p[0].bias == 0.0f, "FP8 scale = amax / 448");
    check(packed[1] == std::byte{0xFE}, "-amax encodes to -448");
  }
  // Constant INT4 group: scale 0, codes 0; all-zero FP8 group: scale 1.
  {
    const float in[4] = {2.5f, 2.5f, 2.5f, 2.5f};
    AffineParams p[1];
    std::byte packed[2] = {std::byte{0xFF}, std::byte{0xFF}};
    check(quantize_reference(QuantFormat::kInt4Packed, in, 4, p, packed) == QuantStatus::kOk &&
              p[0].scale == 0.0f && p[0].bias == 2.5f && packed[0] == std::byte{0} && packed[1] == std::byte{0},
          "constant INT4 group");
    const float z[2] = {0.0f, -0.0f};
    std::byte pk[2];
    check(quantize_reference(QuantFormat::kFp8E5M2, z, 2, std::span(p, 1), pk) == QuantStatus::kOk &&
              p[0].scale == 1.0f,
          "all-zero FP8 group has scale 1");
  }
}

// The argument checks and their order (cpu_quant.hpp:33-42, cpu_dequant.hpp:32-40,
// cuda_dequant.hpp:58-71); outputs untouched on failure.
void argument_checks() {
  std::vector<float> in(16, 1.0f);
  std::vector<AffineParams> p2(2), p1(1);
  std::vector<std::byte> packed(16, std::byte{0x5A});
  const auto untouched = packed;
  auto q = [&](QuantFormat f, std::size_t gs, std::span<AffineParams> p, std::span<std::byte> out) {
    return quantize_reference(f, in, gs, p, out);
  };
  check(q(static_cast<QuantFormat>(4), 8, p2, packed) == QuantStatus::kUnsupportedFormat, "retired INT2");
  check(q(static_cast<QuantFormat>(9), 8, p2, packed) == QuantStatus::kUnsupportedFormat, "unknown format");
  check(q(QuantFormat::kFp8E4M3, 0, p2, packed) == QuantStatus::kInvalidArgument, "FP8 group 0");
  check(q(QuantFormat::kInt4Packed, 3, p2, packed) == QuantStatus::kInvalidArgument, "INT4 odd group");
  check(q(QuantFormat::kFp16, 8, p2, packed) == QuantStatus::kInvalidArgument, "FP16 takes no groups");
  check(q(QuantFormat::kFp8E4M3, 8, p1, packed) == QuantStatus::kInvalidArgument, "params count");
  check(q(QuantFormat::kFp8E4M3, 8, p2, std::span(packed).first(15)) == QuantStatus::kBufferTooSmall,
        "packed too small");
  check(q(QuantFormat::kFp8E4M3, 8, p1, std::span(packed).first(3)) == QuantStatus::kInvalidArgument,
        "params checked before the buffer size");
  in[5] = std::numeric_limits<float>::infinity();
  check(q(QuantFormat::kFp8E4M3, 8, p2, packed) == QuantStatus::kInvalidArgument, "FP8 non-finite input");
  check(q(QuantFormat::kFp16, 0, std::span<AffineParams>(), packed) == QuantStatus::kBufferTooSmall,
        "FP16 needs 2 bytes per value");
  in[5] = 3e38f;
  in[6] = -3e38f;
  check(q(QuantFormat::kInt4Packed, 8, p2, packed) == QuantStatus::kInvalidArgument, "INT4 range overflows");
  check(packed == untouched, "rejected calls leave the output untouched");

  std::vector<float> out(16, 7.0f);
  const std::vector<AffineParams> good(2, AffineParams{1.0f, 0.0f});
  auto d = [&](QuantFormat f, std::size_t n, std::span<const AffineParams> p, std::size_t gs,
               std::span<const std::byte> pk, std::span<float> o) {
    return dequantize_reference(f, pk, n, p, gs, o);
  };
  check(d(static_cast<QuantFormat>(4), 16, good, 8, packed, out) == QuantStatus::kUnsupportedFormat, "dq INT2");
  check(d(QuantFormat::kFp8E4M3, 16, good, 0, packed, out) == QuantStatus::kInvalidArgument, "dq group 0");
  check(d(QuantFormat::kFp8E4M3, 16, std::span(good).first(1), 8, packed, out) == QuantStatus::kInvalidArgument,
        "dq params count");
  const std::vector<AffineParams> biased{{1.0f, 0.0f}, {1.0f, 0.5f}};
  check(d(QuantFormat::kFp8E4M3, 16, biased, 8, packed, out) == QuantStatus::kInvalidArgument, "dq FP8 bias");
  check(d(QuantFormat::kInt4Packed, 16, biased, 8, packed, out) == QuantStatus::kOk, "dq INT4 takes a bias");
  const std::vector<AffineParams> nan{{std::nanf(""), 0.0f}, {1.0f, 0.0f}};
  check(d(QuantFormat::kInt4Packed, 16, nan, 8, packed, out) == QuantStatus::kInvalidArgument, "dq NaN scale");
  std::fill(out.begin(), out.end(), 7.0f);
  check(d(QuantFormat::kFp8E4M3, 16, good, 8, std::span(packed).first(15), out) == QuantStatus::kBufferTooSmall,
        "dq packed too small");
  check(d(QuantFormat::kFp8E4M3, 16, good, 8, packed, std::span(out).first(15)) == QuantStatus::kBufferTooSmall,
        "dq out too small");
  check(std::all_of(out.begin(), out.end(), [](float v) { return v == 7.0f; }), "dq output untouched");
  std::vector<std::uint16_t> h(16);
  check(dequantize_reference_to_fp16(QuantFormat::kFp8E4M3, packed, 16, good, 8, std::span(h).first(15)) ==
            QuantStatus::kBufferTooSmall,
        "dq16 out too small");
  check(dequantize_reference_to_fp16(QuantFormat::kFp16, std::span(packed).first(16), 8, {}, 0, h) ==
            QuantStatus::kOk,
        "dq16 FP16 without parameters");

  using cuda::HostPath;
  const std::vector<std::byte> codes(16);
  const std::vector<AffineParams> one{{1.0f, 0.0f}};
  for (QuantFormat f : {QuantFormat::kFp16, QuantFormat::kInt4Packed, static_cast<QuantFormat>(4)}) {
    check(cuda::emulate_fp8_to_fp16_on_host(f, codes, one, 16, h, HostPath::kScalar) ==
              QuantStatus::kUnsupportedFormat,
          "emulate rejects a non-FP8 format");
  }
  check(cuda::emulate_fp8_to_fp16_on_host(QuantFormat::kFp8E4M3, codes, one, 0, h, HostPath::kScalar) ==
            QuantStatus::kInvalidArgument,
        "emulate group 0");
  check(cuda::emulate_fp8_to_fp16_on_host(QuantFormat::kFp8E4M3, codes, one, 8, h, HostPath::kScalar) ==
            QuantStatus::kInvalidArgument,
        "emulate: two groups need two parameters");
  check(cuda::emulate_fp8_to_fp16_on_host(QuantFormat::kFp8E4M3, codes, one, 16, std::span(h).first(15),
                                          HostPath::kScalar) == QuantStatus::kBufferTooSmall,
        "emulate out too small");
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::printf("usage: test_quant_api <dir>\n");
    return 2;
  }
  const std::string dir = argv[1];
  known_answers();
  argument_checks();

  // Every code decoded (the golden decode tables).
  std::vector<std::uint32_t> d16(65536), d8(256), d5(256);
  for (std::uint32_t c = 0; c < 65536; ++c) d16[c] = bits(decode_fp16(static_cast<std::uint16_t>(c)));
  for (std::uint32_t c = 0; c < 256; ++c) {
    d8[c] = bits(decode_fp8_e4m3(static_cast<std::uint8_t>(c)));
    d5[c] = bits(decode_fp8_e5m2(static_cast<std::uint8_t>(c)));
  }
  write_raw(dir + "/decode_0.bin", d16);
  write_raw(dir + "/decode_1.bin", d8);
  write_raw(dir + "/decode_2.bin", d5);

  // Encodes of the golden inputs.
  const auto x = read_raw<float>(dir + "/encode_in.bin");
  std::vector<std::uint16_t> e16(x.size()), e8(x.size()), e5(x.size());
  for (std::size_t i = 0; i < x.size(); ++i) {
    e16[i] = encode_fp16(x[i]);
    e8[i] = encode_fp8_e4m3(x[i]);
    e5[i] = encode_fp8_e5m2(x[i]);
  }
  write_raw(dir + "/encode_0.bin", e16);
  write_raw(dir + "/encode_1.bin", e8);
  write_raw(dir + "/encode_2.bin", e5);

  // Every FP8 code times every scale of the reference's kernel test, through
  // dequantize_reference_to_fp16 and through both traversals of the host emulation.
  const auto scales = read_raw<float>(dir + "/k_scales.bin");
  std::vector<std::byte> all(256);
  for (int c = 0; c < 256; ++c) all[c] = static_cast<std::byte>(c);
  for (QuantFormat f : {QuantFormat::kFp8E4M3, QuantFormat::kFp8E5M2}) {
    const int fi = static_cast<int>(f);
    std::vector<std::uint16_t> ref_out, scalar_out, vector_out;
    for (float s : scales) {
      const std::vector<AffineParams> p{{s, 0.0f}};
      std::vector<std::uint16_t> a(256), b(256), c(256);
      check(dequantize_reference_to_fp16(f, all, 256, p, 256, a) == QuantStatus::kOk, "fp8 x scale");
      check(cuda::emulate_fp8_to_fp16_on_host(f, all, p, 256, b, cuda::HostPath::kScalar) == QuantStatus::kOk,
            "emulate scalar");
      check(cuda::emulate_fp8_to_fp16_on_host(f, all, p, 256, c, cuda::HostPath::kVector) == QuantStatus::kOk,
            "emulate vector");
      ref_out.insert(ref_out.end(), a.begin(), a.end());
      scalar_out.insert(scalar_out.end(), b.begin(), b.end());
      vector_out.insert(vector_out.end(), c.begin(), c.end());
    }
    write_raw(dir + "/fp8_scales_" + std::to_string(fi) + ".bin", ref_out);
    write_raw(dir + "/emulate_scalar_" + std::to_string(fi) + ".bin", scalar_out);
    write_raw(dir + "/emulate_vector_" + std::to_string(fi) + ".bin", vector_out);
  }

  // Quantize cases: "<format> <group_size> <file>" per line; writes params, packed and the
  // binary16 dequantization of the result.
  std::ifstream cases(dir + "/q_cases.txt");
  int fmt = 0;
  std::size_t gs = 0;
  std::string file;
  while (cases >> fmt >> gs >> file) {
    const auto in = read_raw<float>(dir + "/" + file);
    const QuantFormat f = static_cast<QuantFormat>(fmt);
    std::vector<AffineParams> p(num_groups(in.size(), gs));
    std::vector<std::byte> packed(packed_bytes(f, in.size()));
    check(quantize_reference(f, in, gs, p, packed) == QuantStatus::kOk, "quantize " + file);
    std::vector<std::uint16_t> h(in.size());
    check(dequantize_reference_to_fp16(f, packed, in.size(), p, gs, h) == QuantStatus::kOk, "dq16 " + file);
    std::vector<float> pf;
    for (const AffineParams& a : p) {
      pf.push_back(a.scale);
      pf.push_back(a.bias);
    }
    const std::string tag = std::to_string(fmt) + "_" + std::to_string(gs);
    write_raw(dir + "/q_params_" + tag + ".bin", pf);
    write_raw(dir + "/q_packed_" + tag + ".bin", packed);
    write_raw(dir + "/q_fp16_" + tag + ".bin", h);
  }
  std::printf("%d checks, %d failures\n", g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
