"""Test infrastructure only: the CPU restatement of the reference path (``reax_oracle``) and the recipe
that compiles the reference's own CUDA kernels from their sources into ``oracle/_ref`` (``build_ref``).
The product never imports this package."""
