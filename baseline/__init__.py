# SPDX-License-Identifier: MIT OR Apache-2.0
"""The reference's own CUDA kernels (built from source by baseline/Makefile): the same-GPU bar."""
