"""The reference's `autotune` package path; only its Nsight Compute counter module is on this library's path
(autotune.hw_counters, implemented in cuda_attn.hw_counters). The GPGPU-Sim autotuning study around it is out
of scope."""
