// compat/lora.h — the reference's "lora.h" name (src/fine_tune.cu includes it): the
// LoRA configuration, the global adapter state g_lora and the free functions
// init_lora / lora_forward_all / lora_backward_all / lora_optimizer_step / lora_free
// (src/lora.h:13-20,218-231), acting on the model that last called init().
#pragma once

#include "model.h"

using rubidium::g_lora;
using rubidium::init_lora;
using rubidium::lora_backward_all;
using rubidium::lora_forward_all;
using rubidium::lora_free;
using rubidium::lora_optimizer_step;
using rubidium::LoRAWeights;
