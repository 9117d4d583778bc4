// glsl_runtime.cpp — invocation scheduler for glsl_cpu.hpp (TEST INFRASTRUCTURE ONLY).
#include <barrier>
#include <memory>
#include <thread>
#include <vector>

#include "glsl_cpu.hpp"

namespace glsl {
thread_local uvec3 gl_LocalInvocationID;
thread_local uvec3 gl_GlobalInvocationID;
thread_local uvec3 gl_WorkGroupID;

static std::barrier<>* g_bar = nullptr;

void barrier() { g_bar->arrive_and_wait(); }

static void set_ids(uvec3 local, uvec3 grp, uint lx, uint ly, uint lz) {
  gl_WorkGroupID = grp;
  gl_LocalInvocationID = {lx, ly, lz};
  gl_GlobalInvocationID = {grp.x * local.x + lx, grp.y * local.y + ly, grp.z * local.z + lz};
}

void dispatch(void (*main_fn)(), uvec3 local, uvec3 groups, bool uses_barrier) {
  const uint n = local.x * local.y * local.z;
  for (uint gz = 0; gz < groups.z; ++gz)
    for (uint gy = 0; gy < groups.y; ++gy)
      for (uint gx = 0; gx < groups.x; ++gx) {
        const uvec3 grp = {gx, gy, gz};
        if (!uses_barrier) {
          for (uint i = 0; i < n; ++i) {
            set_ids(local, grp, i % local.x, (i / local.x) % local.y, i / (local.x * local.y));
            main_fn();
          }
          continue;
        }
        // one thread per invocation; a thread that returns early drops out of later barriers
        std::barrier<> bar(static_cast<std::ptrdiff_t>(n));
        g_bar = &bar;
        std::vector<std::thread> ts;
        ts.reserve(n);
        for (uint i = 0; i < n; ++i)
          ts.emplace_back([=, &bar] {
            set_ids(local, grp, i % local.x, (i / local.x) % local.y, i / (local.x * local.y));
            main_fn();
            bar.arrive_and_drop();
          });
        for (auto& t : ts) t.join();
        g_bar = nullptr;
      }
}
}  // namespace glsl
