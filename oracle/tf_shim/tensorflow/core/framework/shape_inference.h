// Shim header: forwards to the single mock of the TF/Eigen types used by the
// reference op sources.  Test infrastructure only.
#pragma once
#include "../../../tf_shim_core.h"
