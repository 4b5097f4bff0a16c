"""cuda-operator-lab for B200: sm_100a kernels behind the reference's Python API.

``cuda_operator_lab.bindings`` mirrors the reference module of the same name;
``cuda_operator_lab.benchmarking`` mirrors its timing helpers;
``cuda_operator_lab.sharding`` adds the multi-GPU (one process per GPU)
partitioning of the large workloads.
"""
