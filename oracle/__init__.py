"""TEST INFRASTRUCTURE: parity oracles of the vox_b200 kernels (see oracle/oracle.py). Not product code."""
