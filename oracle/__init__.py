# SPDX-License-Identifier: MIT OR Apache-2.0
"""TEST INFRASTRUCTURE: the CPU oracle (see oracle.py). Never imported by the product path."""
