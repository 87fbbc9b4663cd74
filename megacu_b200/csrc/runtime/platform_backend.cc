// CUDA platform and peer-table backend host helpers.
//
// Behaviour follows megacu `src/platform/cuda/platform.cc:5-7` (has_stream)
// and `src/backends/nvshmem/backend.cc:5-13` (team_size, has_remote_pes).
#include <megacu/backends/nvshmem.h>
#include <megacu/platform/cuda.h>

namespace megacu::cuda {

bool has_stream(launch_view launch) noexcept { return launch.stream != nullptr; }

}  // namespace megacu::cuda

namespace megacu::nvshmem {

std::int32_t team_size(team_view team) noexcept { return team.team_n_pes; }

bool has_remote_pes(team_view team) noexcept { return team.team_n_pes > 1; }

}  // namespace megacu::nvshmem

extern "C" int megacu_platform_cuda_component() { return 1; }

extern "C" int megacu_backend_nvshmem_component() { return 1; }
