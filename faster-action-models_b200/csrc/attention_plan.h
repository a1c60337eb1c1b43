// Host-side planning shared by the op-level attention entry points.
#pragma once

#include <stddef.h>

#include "../../include/fam.h"
#include "fam_kernels.h"

namespace fam {

struct AttnScratch {
  size_t partial_bytes;   // split partials (O, m, l)
  size_t counter_offset;  // arrival counters after the partials
  size_t counter_bytes;
  size_t total;
};

// Validates the descriptor, chooses the key splits and fills the launch
// arguments (scratch pointers left null) and the scratch layout.
int attention_prepare(const fam_attention_desc* d, AttnArgs* a, AttnScratch* s);
cudaError_t attention_bind_scratch(AttnArgs* a, const AttnScratch& s, void* scratch,
                                   cudaStream_t st);

}  // namespace fam
