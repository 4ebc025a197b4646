import sys

from rusteeze_b200.cli.main import main

sys.exit(main())
