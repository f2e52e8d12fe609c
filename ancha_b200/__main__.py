"""``python -m ancha_b200 separate IN --model PKG -o OUT ...`` (see ancha_b200.cli)."""
import sys

from .cli import main

sys.exit(main())
