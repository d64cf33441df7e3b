"""Command-line front ends: the C++ build_knng_gpu (build_knng_gpu.cpp) and
``python -m knng_gpu_b200.cli`` (multi-GPU via one process per GPU)."""
