"""sm_100a kernels of the eviction hot path behind actkv.kernels' module names."""
