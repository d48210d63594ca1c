# SPDX-License-Identifier: Unlicense
"""CPU oracle of the B200 build (TEST INFRASTRUCTURE ONLY).

Restatements of i.coregistration.opencl's algorithms for the checked path,
used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as
the checker. The product (libcoreg_b200.so) never imports or calls
anything here.
"""
