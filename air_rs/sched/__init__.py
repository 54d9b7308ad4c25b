"""air_rs.sched."""
