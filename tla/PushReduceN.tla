------------------------------ MODULE PushReduceN ------------------------------
(* One block index of the push-reduce engine: N ranks, R rounds, D scratch  *)
(* rounds per (sender, owner). Sender s in round j writes its piece into    *)
(* slot (s, j % D) of every owner -- unless SkipConsumedWait, only once     *)
(* every owner consumed round j - D -- and then publishes filled = j + 1 to *)
(* every owner. Owner q waits until every sender's filled reached j + 1,    *)
(* reads the N - 1 slots (a separate step: senders may act in between) and  *)
(* publishes consumed = j + 1 to every sender.                              *)
EXTENDS Integers

CONSTANTS N, R, D, SkipConsumedWait
VARIABLES sj, sph, rj, rph, filled, consumed, slot, stale
vars == <<sj, sph, rj, rph, filled, consumed, slot, stale>>

Ranks == 0..(N - 1)

Init == /\ sj = [s \in Ranks |-> 0] /\ sph = [s \in Ranks |-> 0]
        /\ rj = [q \in Ranks |-> 0] /\ rph = [q \in Ranks |-> 0]
        /\ filled = [q \in Ranks |-> [s \in Ranks |-> 0]]
        /\ consumed = [s \in Ranks |-> [q \in Ranks |-> 0]]
        /\ slot = [q \in Ranks |-> [s \in Ranks |-> [d \in 0..(D - 1) |-> -1]]]
        /\ stale = FALSE

Write(s) == /\ sj[s] < R /\ sph[s] = 0
            /\ SkipConsumedWait \/ sj[s] < D
               \/ \A q \in Ranks \ {s} : consumed[s][q] >= sj[s] - D + 1
            /\ slot' = [q \in Ranks |-> IF q = s THEN slot[q]
                          ELSE [slot[q] EXCEPT ![s][sj[s] % D] = sj[s]]]
            /\ sph' = [sph EXCEPT ![s] = 1]
            /\ UNCHANGED <<sj, rj, rph, filled, consumed, stale>>

Publish(s) == /\ sj[s] < R /\ sph[s] = 1
              /\ filled' = [q \in Ranks |-> IF q = s THEN filled[q]
                              ELSE [filled[q] EXCEPT ![s] = sj[s] + 1]]
              /\ sj' = [sj EXCEPT ![s] = sj[s] + 1] /\ sph' = [sph EXCEPT ![s] = 0]
              /\ UNCHANGED <<rj, rph, consumed, slot, stale>>

Wait(q) == /\ rj[q] < R /\ rph[q] = 0
           /\ \A s \in Ranks \ {q} : filled[q][s] >= rj[q] + 1
           /\ rph' = [rph EXCEPT ![q] = 1]
           /\ UNCHANGED <<sj, sph, rj, filled, consumed, slot, stale>>

Read(q) == /\ rj[q] < R /\ rph[q] = 1
           /\ stale' = (stale \/ \E s \in Ranks \ {q} : slot[q][s][rj[q] % D] # rj[q])
           /\ rph' = [rph EXCEPT ![q] = 2]
           /\ UNCHANGED <<sj, sph, rj, filled, consumed, slot>>

Consume(q) == /\ rj[q] < R /\ rph[q] = 2
              /\ consumed' = [s \in Ranks |-> IF s = q THEN consumed[s]
                                ELSE [consumed[s] EXCEPT ![q] = rj[q] + 1]]
              /\ rj' = [rj EXCEPT ![q] = rj[q] + 1] /\ rph' = [rph EXCEPT ![q] = 0]
              /\ UNCHANGED <<sj, sph, filled, slot, stale>>

Done == \A r \in Ranks : sj[r] = R /\ rj[r] = R

Next == \/ \E s \in Ranks : Write(s) \/ Publish(s)
        \/ \E q \in Ranks : Wait(q) \/ Read(q) \/ Consume(q)
        \/ (Done /\ UNCHANGED vars)

Spec == Init /\ [][Next]_vars

NoStaleRead == ~stale
=============================================================================
