"""TEST INFRASTRUCTURE ONLY: the CPU oracle (see oracle/oracle.py).  Never imported by winmoe_b200/."""
