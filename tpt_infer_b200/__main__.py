"""``python -m tpt_infer_b200``: the command line (cli.py)."""
import sys

from .cli import main

sys.exit(main())
