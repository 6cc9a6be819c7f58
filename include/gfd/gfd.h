#pragma once
// Host-side umbrella header (same role as the reference include/gfd/gfd.h).
// Device code additionally includes gfd/device.cuh, gfd/warp_spec.cuh or
// gfd/sg_warp_spec.cuh.  The C ABI underneath is include/gfd_b200.h.

#include "gfd/descriptor_queue.h"
#include "gfd/tiled_queue.h"
#include "gfd/sg_task_queue.h"
#include "gfd/copy_engine.h"
#include "gfd/cpu_polling.h"
#include "gfd/warp_spec_session.h"
#include "gfd/staging_pool.h"
#include "gfd/pcie_topology.h"
