// Device-resident state of a model's decode stream: the next input token and
// position, the argmax of the last step, the generated-id counter and the
// step epoch that numbers every exchange word of a step.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace vrt {

struct StepState {
    uint32_t token;
    uint32_t pos;
    uint32_t status;
    uint32_t out_count;
    uint32_t prompt_count;
    uint32_t result_index;
    float result_value;
    uint32_t pad;
    unsigned long long key;
    uint32_t epoch;  // steps run since creation; never reset (exchange sequence numbers)
    uint32_t pad2;
};
// Host writes (reset, prefill start) cover the fields before `epoch`.
constexpr size_t kStepStateHostBytes = offsetof(StepState, epoch);

}  // namespace vrt
