// Grouped, serpentine, optionally persistent tile scheduler shared by host and device.
//
// Produces the same tile order as the reference's SimpleTileScheduler:
//   params_create         tile_scheduler.py:50-78   (group size, tail group, FastDivmods)
//   grid_shape            tile_scheduler.py:110-123 (persistent: (cm, cn, clusters per wave))
//   map_cluster           tile_scheduler.py:125-146 (linear cluster id -> cluster (m, n))
//   first / next work id  tile_scheduler.py:94-107, :175-183 (start at blockIdx.z or the linear
//                         cluster id; persistent stride gridDim.z)
//   valid                 tile_scheduler.py:159-165
// The batch (L) coordinate is fixed at 0 as in the reference (tile_scheduler.py:96).
#pragma once
#include "fast_divmod.h"

namespace cpg {

enum RasterOrder : int32_t { kAlongM = 0, kAlongN = 1 };

struct SchedParams {
  int32_t ncluster_m, ncluster_n, ncluster_l;
  int32_t raster_order;
  FastDivmod dm_clusters_per_problem;
  int32_t num_groups_regular;
  FastDivmod dm_group_size;
  FastDivmod dm_group_size_tail;
  FastDivmod dm_num_clusters_in_group;
  int32_t cluster_m, cluster_n;
  int32_t is_persistent;
};

CPG_HD int32_t ceil_div_i32(int32_t a, int32_t b) { return (a + b - 1) / b; }

// tile_scheduler.py:50-78.  All counts must be >= 1.
CPG_HD SchedParams sched_params_create(int32_t ntiles_m, int32_t ntiles_n, int32_t ntiles_l,
                                       int32_t raster_order, int32_t group_size,
                                       int32_t cluster_m, int32_t cluster_n, int32_t is_persistent) {
  SchedParams p;
  p.ncluster_m = ceil_div_i32(ntiles_m, cluster_m);
  p.ncluster_n = ceil_div_i32(ntiles_n, cluster_n);
  p.ncluster_l = ntiles_l;
  p.raster_order = raster_order;
  int32_t clusters_per_problem = p.ncluster_m * p.ncluster_n;
  int32_t nfast = raster_order == kAlongM ? p.ncluster_m : p.ncluster_n;
  int32_t nslow = raster_order == kAlongM ? p.ncluster_n : p.ncluster_m;
  int32_t g = group_size < nfast ? group_size : nfast;
  int32_t tail = nfast % g;
  p.num_groups_regular = nfast / g;
  p.dm_clusters_per_problem = fast_divmod_create(clusters_per_problem);
  p.dm_group_size = fast_divmod_create(g);
  p.dm_group_size_tail = fast_divmod_create(tail > 0 ? tail : 1);
  p.dm_num_clusters_in_group = fast_divmod_create(g * nslow);
  p.cluster_m = cluster_m;
  p.cluster_n = cluster_n;
  p.is_persistent = is_persistent;
  return p;
}

// tile_scheduler.py:110-123.
CPG_HD void sched_grid_shape(const SchedParams& p, int32_t max_active_clusters, int32_t grid[3]) {
  int32_t cx = p.ncluster_m * p.cluster_m;
  int32_t cy = p.ncluster_n * p.cluster_n;
  int32_t cz = p.ncluster_l;
  if (!p.is_persistent) {
    grid[0] = cx; grid[1] = cy; grid[2] = cz;
    return;
  }
  int64_t in_problem = int64_t(cx) * cy * cz;
  int64_t in_cluster = int64_t(p.cluster_m) * p.cluster_n;
  int64_t per_wave = int64_t(max_active_clusters) * in_cluster;
  int64_t persistent_ctas = in_problem < per_wave ? in_problem : per_wave;
  grid[0] = p.cluster_m;
  grid[1] = p.cluster_n;
  grid[2] = static_cast<int32_t>(persistent_ctas / in_cluster);
}

// tile_scheduler.py:125-146: linear cluster id -> (cluster_m, cluster_n).
CPG_HD void sched_map_cluster(const SchedParams& p, int32_t cluster_id, int32_t& cid_m,
                              int32_t& cid_n) {
  int32_t group_id, id_in_group, slow, fast_in_group;
  fast_divmod(p.dm_num_clusters_in_group, cluster_id, group_id, id_in_group);
  if (group_id < p.num_groups_regular) {
    fast_divmod(p.dm_group_size, id_in_group, slow, fast_in_group);
  } else {
    fast_divmod(p.dm_group_size_tail, id_in_group, slow, fast_in_group);
  }
  if (group_id % 2 == 1) {
    int32_t nslow = p.raster_order == kAlongM ? p.ncluster_n : p.ncluster_m;
    slow = nslow - 1 - slow;
  }
  int32_t fast = group_id * p.dm_group_size.divisor + fast_in_group;
  if (p.raster_order == kAlongN) {
    cid_m = slow; cid_n = fast;
  } else {
    cid_m = fast; cid_n = slow;
  }
}

CPG_HD int32_t sched_total_clusters(const SchedParams& p) {
  return p.ncluster_m * p.ncluster_n * p.ncluster_l;
}

}  // namespace cpg
