"""Native sources of libkernelo_b200 and the script that builds it."""
