// Launch metadata for every exported kernel, as JSON with the keys of the
// reference's AOTResult.to_metadata() (src/neso/aot_compile.py:108-117):
//   kernel_name, params[{index, name, type, metal_type, is_pointer}],
//   constants, threadgroup_size, num_warps, grid
// Parameter entries follow KernelParameter (src/neso/backend/abi.py:19-27);
// `metal_type` carries the C type of the argument so consumers written against
// the reference schema keep working, and `cuda_type` repeats it explicitly.
// threadgroup_size / num_warps report the CTA this library actually launches.
#include <cstring>
#include <string>
#include <unordered_map>

#include "runtime.h"

namespace neso {
namespace {

struct Param {
  const char* name;
  const char* type;   // Triton signature type, e.g. "*fp16", "i32", "fp32"
  const char* ctype;  // C type of the argument
};

struct KernelMeta {
  const char* name;
  std::initializer_list<Param> params;
  const char* constants;  // JSON object text
  int threads;
  const char* grid[3];
};

std::string to_json(const KernelMeta& k) {
  std::string s = "{\"kernel_name\": \"";
  s += k.name;
  s += "\", \"params\": [";
  int i = 0;
  for (const Param& p : k.params) {
    if (i) s += ", ";
    const bool ptr = p.type[0] == '*';
    s += "{\"index\": " + std::to_string(i) + ", \"name\": \"" + p.name + "\", \"type\": \"" + p.type +
         "\", \"metal_type\": \"" + p.ctype + "\", \"cuda_type\": \"" + p.ctype +
         "\", \"is_pointer\": " + (ptr ? "true" : "false") + "}";
    ++i;
  }
  s += "], \"constants\": ";
  s += k.constants;
  s += ", \"threadgroup_size\": " + std::to_string(k.threads);
  s += ", \"num_warps\": " + std::to_string(k.threads / 32);
  s += ", \"grid\": [\"" + std::string(k.grid[0]) + "\", \"" + k.grid[1] + "\", \"" + k.grid[2] + "\"]}";
  return s;
}

const std::unordered_map<std::string, std::string>& table() {
  static const std::unordered_map<std::string, std::string> t = [] {
    const char* F16P = "const __half*";
    const KernelMeta ks[] = {
        {"vector_add",
         {{"x", "*fp32", "const float*"}, {"y", "*fp32", "const float*"}, {"output", "*fp32", "float*"},
          {"n_elements", "i32", "int32_t"}},
         "{\"BLOCK_SIZE\": 1024}", 256, {"cdiv(n_elements, BLOCK_SIZE)", "1", "1"}},
        {"add_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"y_ptr", "*fp32", "const float*"}, {"z_ptr", "*fp32", "float*"},
          {"n_elements", "i32", "int32_t"}},
         "{\"BLOCK_SIZE\": 1024}", 256, {"cdiv(n_elements, BLOCK_SIZE)", "1", "1"}},
        {"scale",
         {{"x", "*fp32", "const float*"}, {"output", "*fp32", "float*"}, {"factor", "fp32", "float"},
          {"n_elements", "i32", "int32_t"}},
         "{\"BLOCK_SIZE\": 1024}", 256, {"cdiv(n_elements, BLOCK_SIZE)", "1", "1"}},
        {"flash_attention_fwd",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"O", "*fp32", "float*"},
          {"N", "i32", "int32_t"}, {"stride_qo", "i32", "int32_t"}, {"stride_kv", "i32", "int32_t"},
          {"scale", "fp32", "float"}},
         "{\"d\": 64, \"BM\": 128, \"BN\": 128}", 384, {"N / BM", "1", "1"}},
        {"rel_pos_fa2_fwd",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"bias", "*fp16", F16P},
          {"O", "*fp16", "__half*"}, {"T", "i32", "int32_t"}, {"stride", "i32", "int32_t"},
          {"scale", "fp32", "float"}, {"stride_h", "i32", "int32_t"}, {"bias_stride_h", "i32", "int32_t"}},
         "{\"d\": 128, \"BM\": 128, \"BN\": 128}", 384, {"T / BM", "nh", "1"}},
        {"fa2_fwd",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"O", "*fp32", "float*"},
          {"B", "i32", "int32_t"}, {"H", "i32", "int32_t"}, {"S", "i32", "int32_t"}, {"D", "i32", "int32_t"},
          {"scale", "fp32", "float"}, {"causal", "i32", "int32_t"}},
         "{}", 384, {"cdiv(S, 256)", "B * H", "1"}},
        // MSL FA2 kernels (fp16 io_type shown; use_half = 0 takes fp32 buffers).
        {"flash_attention_fwd_msl",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"O", "*fp16", "__half*"},
          {"N", "i32", "int32_t"}, {"d_head", "i32", "int32_t"}, {"scale", "fp32", "float"}},
         "{\"BM\": 32, \"BN\": 32, \"d\": 64, \"THREADS\": 1024, \"use_half\": 1}", 384, {"N / BM", "1", "1"}},
        {"flash_attention_opt",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"O", "*fp16", "__half*"},
          {"N", "i32", "int32_t"}, {"d_head", "i32", "int32_t"}, {"scale", "fp32", "float"}},
         "{\"BM\": 32, \"BN\": 32, \"d\": 64, \"THREADS\": 1024, \"use_half\": 1}", 384, {"N / BM", "1", "1"}},
        {"flash_attention_d128",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"O", "*fp16", "__half*"},
          {"N", "i32", "int32_t"}, {"d_head", "i32", "int32_t"}, {"scale", "fp32", "float"}},
         "{\"BM\": 32, \"BN\": 32, \"d\": 128, \"THREADS\": 1024, \"use_half\": 1}", 384,
         {"N / BM", "1", "1"}},
        {"fa2_fwd_relpos_table",
         {{"Q", "*fp16", F16P}, {"K", "*fp16", F16P}, {"V", "*fp16", F16P}, {"table", "*fp32", "const float*"},
          {"O", "*fp32", "float*"}, {"B", "i32", "int32_t"}, {"H", "i32", "int32_t"}, {"S", "i32", "int32_t"},
          {"D", "i32", "int32_t"}, {"scale", "fp32", "float"}, {"causal", "i32", "int32_t"}},
         "{}", 384, {"cdiv(S, 256)", "B * H", "1"}},
        {"matmul_kernel",
         {{"a_ptr", "*fp16", F16P}, {"b_ptr", "*fp16", F16P}, {"c_ptr", "*fp32", "float*"}, {"M", "i32", "int32_t"},
          {"N", "i32", "int32_t"}, {"K", "i32", "int32_t"}, {"stride_am", "i32", "int32_t"},
          {"stride_ak", "i32", "int32_t"}, {"stride_bk", "i32", "int32_t"}, {"stride_bn", "i32", "int32_t"},
          {"stride_cm", "i32", "int32_t"}, {"stride_cn", "i32", "int32_t"}},
         "{\"BLOCK_M\": 128, \"BLOCK_N\": 128, \"BLOCK_K\": 32}", 256,
         {"cdiv(M, BLOCK_M)", "cdiv(N, BLOCK_N)", "1"}},
        {"matmul_tiled",
         {{"a", "*fp16", F16P}, {"b", "*fp16", F16P}, {"c", "*fp32", "float*"}, {"K", "i32", "int32_t"},
          {"stride_am", "i32", "int32_t"}, {"stride_bk", "i32", "int32_t"}, {"stride_cm", "i32", "int32_t"}},
         "{\"BM\": 128, \"BN\": 128}", 256, {"M / BM", "N / BN", "1"}},
        {"w8a16_matmul",
         {{"A", "*fp16", F16P}, {"B", "*i8", "const int8_t*"}, {"C", "*fp32", "float*"}, {"K", "i32", "int32_t"},
          {"stride_am", "i32", "int32_t"}, {"stride_bk", "i32", "int32_t"}, {"stride_cm", "i32", "int32_t"}},
         "{\"BM\": 128, \"BN\": 128, \"BK\": 64}", 512, {"cdiv(M, BM)", "cdiv(N, BN)", "1"}},
        {"w8a16_scaled_matmul",
         {{"A", "*fp16", F16P}, {"B", "*i8", "const int8_t*"}, {"C", "*fp32", "float*"},
          {"scale", "*fp16", F16P}, {"K", "i32", "int32_t"}, {"stride_am", "i32", "int32_t"},
          {"stride_bk", "i32", "int32_t"}, {"stride_cm", "i32", "int32_t"}},
         "{\"BM\": 128, \"BN\": 128, \"BK\": 64}", 512, {"cdiv(M, BM)", "cdiv(N, BN)", "1"}},
        {"w8a16_matmul_kernel",
         {{"a_ptr", "*fp16", F16P}, {"b_int8_ptr", "*i8", "const int8_t*"}, {"c_ptr", "*fp32", "float*"},
          {"scale_ptr", "*fp32", "const float*"}, {"M", "i32", "int32_t"}, {"N", "i32", "int32_t"},
          {"K", "i32", "int32_t"}, {"stride_am", "i32", "int32_t"}, {"stride_ak", "i32", "int32_t"},
          {"stride_bk", "i32", "int32_t"}, {"stride_bn", "i32", "int32_t"}, {"stride_cm", "i32", "int32_t"},
          {"stride_cn", "i32", "int32_t"}},
         "{\"BLOCK_M\": 32, \"BLOCK_N\": 32, \"BLOCK_K\": 32}", 512,
         {"cdiv(M, BLOCK_M)", "cdiv(N, BLOCK_N)", "1"}},
        {"w8a16_matmul_mnk",
         {{"X", "*fp16", F16P}, {"W", "*i8", "const int8_t*"}, {"scale", "*fp16", F16P}, {"Y", "*fp32", "float*"},
          {"M", "i32", "int32_t"}, {"N", "i32", "int32_t"}, {"K", "i32", "int32_t"}},
         "{}", 512, {"internal", "1", "1"}},
        {"w4a16_g128_matmul",
         {{"X", "*fp16", F16P}, {"Wq", "*u8", "const uint8_t*"}, {"scales", "*fp16", F16P},
          {"Y", "*fp32", "float*"}, {"M", "i32", "int32_t"}, {"N", "i32", "int32_t"}, {"K", "i32", "int32_t"}},
         "{\"GROUP\": 128}", 512, {"internal", "1", "1"}},
        {"rmsnorm_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"weight_ptr", "*fp32", "const float*"}, {"out_ptr", "*fp32", "float*"},
          {"row_stride", "i32", "int32_t"}, {"n_cols", "i32", "int32_t"}, {"eps", "fp32", "float"}},
         "{\"BLOCK_SIZE\": 128}", 256, {"M", "1", "1"}},
        {"residual_rmsnorm_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"residual_ptr", "*fp32", "const float*"},
          {"weight_ptr", "*fp32", "const float*"}, {"out_ptr", "*fp32", "float*"}, {"row_stride", "i32", "int32_t"},
          {"n_cols", "i32", "int32_t"}, {"eps", "fp32", "float"}},
         "{\"BLOCK_SIZE\": 128}", 256, {"M", "1", "1"}},
        {"rope_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"cos_ptr", "*fp32", "const float*"}, {"sin_ptr", "*fp32", "const float*"},
          {"out_ptr", "*fp32", "float*"}, {"seq_len", "i32", "int32_t"}, {"head_dim", "i32", "int32_t"}},
         "{\"BLOCK_D\": 32}", 256, {"seq_len", "1", "1"}},
        {"silu_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"out_ptr", "*fp32", "float*"}, {"n", "i32", "int32_t"}},
         "{\"BLOCK\": 256}", 256, {"cdiv(n, BLOCK)", "1", "1"}},
        {"softmax_kernel",
         {{"output_ptr", "*fp32", "float*"}, {"input_ptr", "*fp32", "const float*"},
          {"input_row_stride", "i32", "int32_t"}, {"output_row_stride", "i32", "int32_t"}, {"n_cols", "i32", "int32_t"}},
         "{\"BLOCK_SIZE\": 128}", 256, {"M", "1", "1"}},
        {"per_channel_dequant_kernel",
         {{"x_int8_ptr", "*i32", "const int32_t*"}, {"scale_ptr", "*fp32", "const float*"},
          {"zero_ptr", "*fp32", "const float*"}, {"out_ptr", "*fp32", "float*"}, {"n_rows", "i32", "int32_t"},
          {"n_cols", "i32", "int32_t"}},
         "{\"BLOCK_M\": 32, \"BLOCK_N\": 32}", 256, {"cdiv(n_rows, BLOCK_M)", "cdiv(n_cols, BLOCK_N)", "1"}},
        {"grouped_dequant_kernel",
         {{"x_int8_ptr", "*i32", "const int32_t*"}, {"scale_ptr", "*fp32", "const float*"},
          {"zero_ptr", "*fp32", "const float*"}, {"out_ptr", "*fp32", "float*"}, {"n", "i32", "int32_t"},
          {"group_size", "i32", "int32_t"}},
         "{\"BLOCK\": 256}", 256, {"cdiv(n, BLOCK)", "1", "1"}},
        {"quantize_kernel",
         {{"x_ptr", "*fp32", "const float*"}, {"scale_ptr", "*fp32", "const float*"}, {"out_ptr", "*i32", "int32_t*"},
          {"n", "i32", "int32_t"}},
         "{\"BLOCK\": 256}", 256, {"cdiv(n, BLOCK)", "1", "1"}},
    };
    std::unordered_map<std::string, std::string> m;
    for (const KernelMeta& k : ks) m.emplace(k.name, to_json(k));
    return m;
  }();
  return t;
}

}  // namespace
}  // namespace neso

extern "C" const char* neso_kernel_metadata(const char* kernel_name) {
  if (kernel_name == nullptr) return nullptr;
  const auto& t = neso::table();
  auto it = t.find(kernel_name);
  return it == t.end() ? nullptr : it->second.c_str();
}
