"""`python -m mlx_batch_invariant_b200 verify` (see _cli.py)."""

import sys

from ._cli import main

sys.exit(main())
