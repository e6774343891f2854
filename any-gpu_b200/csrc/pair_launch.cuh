// Host launcher of the CTA-pair tcgen05 kernel (umma2_kernel.cuh) shared by
// the GEMM and conv2d paths: one cluster of 2 CTAs per pair of SMs, at most
// one per tile.
#pragma once

#include <algorithm>

#include "agpu_internal.cuh"
#include "umma2_kernel.cuh"

namespace agpu {

template <class P>
agpu_status launch_pair(agpu_device* dev, const CUtensorMap& ta, const CUtensorMap& tb,
                        const P& pol, long long tiles, cudaStream_t s, const char* what) {
  using Cfg = umma::PairCfg<P::BN, P::EPI_EXTRA>;
  auto kern = umma::umma_tf32_pair_kernel<P>;
  AGPU_CUDA(set_smem_once<umma::umma_tf32_pair_kernel<P>>(dev, Cfg::SMEM));
  const long long clusters = std::min<long long>(tiles, std::max(1, dev->sm_count / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // may start its prologue while the previous kernel drains (the kernel
  // waits on griddepcontrol before touching global memory)
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  AGPU_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, pol, dev->d_status));
  return after_launch(dev, what);
}

}  // namespace agpu
