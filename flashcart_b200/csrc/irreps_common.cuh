// Direction-tensor (edge attribute) kernels: shared includes.
#pragma once
#include "fc_base.cuh"
