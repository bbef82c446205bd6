"""siliconfer_b200 -- siliconfer's Q4Linear int4 path on NVIDIA B200 (sm_100a).

Public surface:
  siliconfer_b200.kernels.cuda   -- mirror of siliconfer.kernels.neon
  siliconfer_b200.q4_linear      -- Q4Linear (torch.nn.Module)
  siliconfer_b200.q4_loader      -- _pack_and_replace_linears
  siliconfer_b200.quant          -- packers (host and device)
  siliconfer_b200.tensor_parallel-- column/row-parallel Q4Linear over NCCL
The compute lives in libsf_q4.so (C ABI: include/sf_q4.h).
"""
__version__ = "0.1.0"
