// Declarations shared by the simulation kernels and the Python bindings.
#pragma once

#include <cuda_runtime.h>
#include <vector>

#include "planner.h"
#include "rules.h"
#include "sense.h"

namespace ad {

size_t tick_smem_bytes();
void phase_profile_enable(bool on);
std::vector<unsigned long long> phase_profile_read();
std::vector<unsigned long long> sense_profile_read();
std::vector<unsigned long long> plan_profile_read();
size_t plan_smem_bytes(const SimParams& sp);
size_t sense_smem_bytes(const SimParams& sp);
void validate_params(const SimParams& sp);

void launch_control(const World& w, const SimParams& sp, const int32_t* actions, cudaStream_t st);
void launch_plan(const World& w, const SimParams& sp, int force, cudaStream_t st);
void launch_tick(const World& w, const SimParams& sp, uint32_t tick, int run_game, int threads, cudaStream_t st);
void launch_physics(const World& w, const SimParams& sp, int ticks, int threads, cudaStream_t st);
void launch_observe(const World& w, const SimParams& sp, cudaStream_t st);
void launch_perceive(const World& w, const SimParams& sp, int threads, cudaStream_t st);
void launch_sense(const World& w, const SimParams& sp, int force, cudaStream_t st);

void host_control(World w, const SimParams& sp, const int32_t* actions);
void host_plan(World w, const SimParams& sp, int force);
void host_tick(World w, const SimParams& sp, uint32_t tick, int run_game);
void host_physics(World w, const SimParams& sp, int ticks);
void host_observe(World w, const SimParams& sp);
void host_perceive(World w, const SimParams& sp);
void host_sense(World w, const SimParams& sp, int force);

}  // namespace ad
