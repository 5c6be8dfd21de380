"""``python -m kernelo_b200``: the command line interface (see :mod:`kernelo_b200.cli`)."""

import sys

from kernelo_b200.cli import main

sys.exit(main())
