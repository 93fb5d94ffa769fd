// Host build of the chunk kernel's triangular inverse (tri_inverse64 in csrc/chunk_tc.cu) for a CPU test.
//
// The test cuts the device function out of the kernel source into the file named by INV_INC and
// compiles it here with stand-ins for the CUDA pieces it uses: shared-memory loads become plain loads,
// the intra group's named barrier becomes a std::barrier over 256 threads and __syncwarp a barrier over
// the 32 threads of the caller's warp.  fmaf is the host's correctly rounded fused multiply-add, as on
// the GPU, so the result is the device's up to the order of operations the kernel fixes.
//
// Usage: host_inverse X.bin T.bin   (X.bin: 64 x 64 float32 strictly lower X, row-major; T.bin receives
// the 64 x 64 result the 256 threads leave in place of X).
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <thread>
#include <vector>

#define __device__
#define __forceinline__ inline
struct float4 {
  float x, y, z, w;
};
struct float2 {
  float x, y;
};
static inline float4 make_float4(float a, float b, float c, float d) { return {a, b, c, d}; }
static inline float2 make_float2(float a, float b) { return {a, b}; }
constexpr int LT = 68, LP = 36;  // the kernel's row strides of the inverse scratch and the merge scratch
static inline float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }
static inline float2 lds2(const float* p) { return {p[0], p[1]}; }
static inline float lds1(const float* p) { return *p; }
static inline float f4get(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
static std::barrier<>* g_group;
static std::barrier<>* g_warp[8];
thread_local int t_warp;
static inline void group_sync(int) { g_group->arrive_and_wait(); }
static inline void __syncwarp() { g_warp[t_warp]->arrive_and_wait(); }

#include INV_INC

int main(int argc, char** argv) {
  if (argc != 3) return 2;
  std::vector<float> buf(64 * LT + 32 * LP + 16, 0.f);
  float* X = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(buf.data()) + 15) & ~uintptr_t(15));
  float* P = X + 64 * LT;
  FILE* f = std::fopen(argv[1], "rb");
  if (!f) return 3;
  for (int i = 0; i < 64; ++i)
    if (std::fread(X + i * LT, 4, 64, f) != 64) return 4;
  std::fclose(f);
  std::barrier<> group(256);
  g_group = &group;
  for (int w = 0; w < 8; ++w) g_warp[w] = new std::barrier<>(32);
  std::vector<std::thread> th;
  for (int t = 0; t < 256; ++t)
    th.emplace_back([=] {
      t_warp = t >> 5;
      tri_inverse64(X, P, t >> 5, t & 31);
    });
  for (auto& t : th) t.join();
  for (int w = 0; w < 8; ++w) delete g_warp[w];
  f = std::fopen(argv[2], "wb");
  if (!f) return 5;
  for (int i = 0; i < 64; ++i) std::fwrite(X + i * LT, 4, 64, f);
  std::fclose(f);
  return 0;
}
