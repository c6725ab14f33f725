"""`python -m enzyme_b200 kernels/<name> --sizes ...` (the `axon` command)."""

from .cli import main

main()
