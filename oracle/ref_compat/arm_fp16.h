/* The reference includes <arm_fp16.h>; the types it needs live in arm_neon.h here. */
#pragma once
#include "arm_neon.h"
