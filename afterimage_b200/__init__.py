"""afterimage_b200: lossless BF16 weight reconstruction for Afterimage
stores on B200 (sm_100a).

`afterimage_b200.runtime` holds the modules that replace the reference's
`afterimage.runtime` ones (codec, decoders, store, planner, engine, verify)
plus the tensor-parallel decoder. The CUDA kernels and the C ABI are in
`afterimage_b200/csrc` and build into `afterimage_b200/lib/libafterimage_b200.so`
(`python -m afterimage_b200.csrc.build`).
"""
