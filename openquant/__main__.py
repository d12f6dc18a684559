"""python -m openquant ... == the `openquant` command."""
from openquant_b200.cli import main

raise SystemExit(main())
