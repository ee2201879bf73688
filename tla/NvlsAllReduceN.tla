---------------------------- MODULE NvlsAllReduceN ----------------------------
(* One block index of the NVLS AllReduce: N ranks, R rounds, B round       *)
(* buffers of N slices per rank. Copier of rank r, step s (0..R+1), two     *)
(* actions: CopyIn (when s < R, copy input round s into buffer s % B, then  *)
(* publish s + 1) and CopyOut (when s >= 2, wait until every mover          *)
(* published s - 1 and copy buffer (s-2) % B out: every slice must hold     *)
(* round s-2 reduced). The kernel's order is CopyOut first; with InFirst   *)
(* CopyIn comes first (an order that holds here but failed on the GPU).     *)
(* With Ahead (the kernel's opt-in for a buffer per round) the copier       *)
(* copies every round in first (steps 0..R-1), then round s - R out at     *)
(* step s after every mover published s - R + 1.                          *)
(* Mover of rank r, step s < R: waits until every copier published s + 1   *)
(* (only its own when not MoverWaitsAll), reads slice r of buffer s % B on  *)
(* every rank (the switch's ld_reduce: must hold round s input), then       *)
(* writes the reduced slice r into every rank's buffer (the multicast store) *)
(* and publishes s + 1. Reading and writing are separate steps.            *)
EXTENDS Integers

CONSTANTS N, R, B, MoverWaitsAll, InFirst, Ahead
VARIABLES cs, cph, ms, mph, cflag, mflag, buf, bad
vars == <<cs, cph, ms, mph, cflag, mflag, buf, bad>>

Ranks == 0..(N - 1)
Empty == <<-1, -1>>

Init == /\ cs = [r \in Ranks |-> 0] /\ cph = [r \in Ranks |-> 0]
        /\ ms = [r \in Ranks |-> 0] /\ mph = [r \in Ranks |-> 0]
        /\ cflag = [r \in Ranks |-> 0] /\ mflag = [r \in Ranks |-> 0]
        /\ buf = [r \in Ranks |-> [b \in 0..(B - 1) |-> [q \in Ranks |-> Empty]]]
        /\ bad = FALSE

\* The phase of the step each copier action takes, and what follows it.
OutPhase == IF InFirst THEN 1 ELSE 0
InPhase == IF InFirst THEN 0 ELSE 1

CopyOut(r) == LET s == cs[r] IN
              /\ ~Ahead /\ s < R + 2 /\ cph[r] = OutPhase
              /\ s >= 2 => \A q \in Ranks : mflag[q] >= s - 1
              /\ bad' = (bad \/ (s >= 2 /\ \E q \in Ranks : buf[r][(s - 2) % B][q] # <<s - 2, 1>>))
              /\ IF InFirst THEN cs' = [cs EXCEPT ![r] = s + 1] /\ cph' = [cph EXCEPT ![r] = 0]
                 ELSE UNCHANGED cs /\ cph' = [cph EXCEPT ![r] = 1]
              /\ UNCHANGED <<ms, mph, cflag, mflag, buf>>

CopyInPublish(r) == LET s == cs[r] IN
                    /\ ~Ahead /\ s < R + 2 /\ cph[r] = InPhase
                    /\ buf' = IF s < R THEN [buf EXCEPT ![r][s % B] = [q \in Ranks |-> <<s, 0>>]]
                              ELSE buf
                    /\ IF InFirst THEN UNCHANGED cs /\ cph' = [cph EXCEPT ![r] = 1]
                       ELSE cs' = [cs EXCEPT ![r] = s + 1] /\ cph' = [cph EXCEPT ![r] = 0]
                    /\ cflag' = [cflag EXCEPT ![r] = s + 1]
                    /\ UNCHANGED <<ms, mph, mflag, bad>>

CopyAhead(r) == LET s == cs[r] IN
                /\ Ahead /\ s < 2 * R
                /\ IF s < R
                      THEN /\ buf' = [buf EXCEPT ![r][s % B] = [q \in Ranks |-> <<s, 0>>]]
                           /\ cflag' = [cflag EXCEPT ![r] = s + 1]
                           /\ UNCHANGED bad
                      ELSE /\ \A q \in Ranks : mflag[q] >= s - R + 1
                           /\ bad' = (bad \/ \E q \in Ranks : buf[r][(s - R) % B][q] # <<s - R, 1>>)
                           /\ UNCHANGED <<buf, cflag>>
                /\ cs' = [cs EXCEPT ![r] = s + 1]
                /\ UNCHANGED <<cph, ms, mph, mflag>>

MoverWait(r) == LET s == ms[r] IN
                /\ s < R /\ mph[r] = 0
                /\ IF MoverWaitsAll THEN \A q \in Ranks : cflag[q] >= s + 1 ELSE cflag[r] >= s + 1
                /\ mph' = [mph EXCEPT ![r] = 1]
                /\ UNCHANGED <<cs, cph, ms, cflag, mflag, buf, bad>>

MoverRead(r) == LET s == ms[r] IN
                /\ s < R /\ mph[r] = 1
                /\ bad' = (bad \/ \E q \in Ranks : buf[q][s % B][r] # <<s, 0>>)
                /\ mph' = [mph EXCEPT ![r] = 2]
                /\ UNCHANGED <<cs, cph, ms, cflag, mflag, buf>>

MoverWrite(r) == LET s == ms[r] IN
                 /\ s < R /\ mph[r] = 2
                 /\ buf' = [q \in Ranks |-> [buf[q] EXCEPT ![s % B][r] = <<s, 1>>]]
                 /\ ms' = [ms EXCEPT ![r] = s + 1] /\ mph' = [mph EXCEPT ![r] = 0]
                 /\ mflag' = [mflag EXCEPT ![r] = s + 1]
                 /\ UNCHANGED <<cs, cph, cflag, bad>>

Done == \A r \in Ranks : cs[r] = (IF Ahead THEN 2 * R ELSE R + 2) /\ ms[r] = R

Next == \/ \E r \in Ranks : CopyOut(r) \/ CopyInPublish(r) \/ CopyAhead(r) \/ MoverWait(r) \/ MoverRead(r)
                            \/ MoverWrite(r)
        \/ (Done /\ UNCHANGED vars)

Spec == Init /\ [][Next]_vars

RoundsInOrder == ~bad
=============================================================================
