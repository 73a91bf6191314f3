// capi_internal.h -- what the control plane (runtime.cu) needs from the npu_* layer (capi.cu)
#pragma once

#include <string>

struct NpuModel;

// npu_model_load with the model's device chosen: the model's buffers, kernels and streams live on
// CUDA device `ordinal`.  NULL on failure, with the message for npu_last_error on this thread.
NpuModel *npu_model_load_on(const char *scenario_path, int ordinal);

// set the calling thread's npu_last_error message
void npu_set_last_error(const std::string &msg);
