"""Reference-compatible module namespace (`src.gpu_cache`, `src.gpu_kernels`,
`src.gpu_ops`, `src.inference`) backed by the sm_100a kernels of libdkv.so."""
