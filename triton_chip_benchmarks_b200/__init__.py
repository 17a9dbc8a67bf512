"""B200-native (sm_100a) chip peak-throughput probes.

Hand-written CUDA kernels in ``libtcb.so`` (C ABI in ``include/tcb.h``) for the
three measurement paths of the chip metric suite - the resident-operand
tensor probe, the vector FMA-chain probe and the device copy/read bandwidth
probe - with Python drivers that keep the suite's 17-row JSON contract:

* ``python -m triton_chip_benchmarks_b200.bench_suite``     full table
* ``python -m triton_chip_benchmarks_b200.bench_tensor``    tensor rows
* ``python -m triton_chip_benchmarks_b200.bench_vector``    vector rows
* ``python -m triton_chip_benchmarks_b200.bench_bandwidth`` bandwidth row
* ``python -m triton_chip_benchmarks_b200.replicas``        N-GPU concurrent replicas
"""

__version__ = "0.1.0"
