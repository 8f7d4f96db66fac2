# SPDX-License-Identifier: MIT
"""TEST INFRASTRUCTURE ONLY: CPU checkers of the CUDA engine (see oracle.py)."""
